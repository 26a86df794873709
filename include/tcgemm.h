/*
 * tcgemm.h -- C ABI of the B200 (sm_100a) tensor-core GEMM library
 * (libtcgemm.so).  Plain pointers and sizes; no C++ or torch types.
 *
 * Every entry point computes C = A * B for `batches` independent problems,
 * overwriting C (alpha = 1, beta = 0), and is asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream).  The caller owns every
 * buffer; the library allocates nothing except where an entry point says so.
 *
 * Layouts (row-major, batch b at offset b * rows * cols of each operand):
 *   A  : M x K, K contiguous
 *   B  : TCG_B_KN -> K x N (N contiguous)      [reference fp16 contract]
 *        TCG_B_NK -> N x K, "BT" (K contiguous) [reference int8/int4 contract]
 *   C  : M x N, N contiguous, 4-byte elements (float or int32)
 * int4 operands are packed two per byte along K, low nibble = even k,
 * K/2 bytes per row (reference src/data_int4.h:4-6).
 *
 * Shape and alignment rules (TCG_ERR_SHAPE / TCG_ERR_ALIGN otherwise): each
 * TMA-loaded row must be a multiple of 16 bytes and A, B must be 16-byte
 * aligned:  fp16 K % 8 == 0 (and N % 8 == 0 for TCG_B_KN); int8 K % 16 == 0
 * (N % 16 == 0 for TCG_B_KN); int4 K % 32 == 0.  M and N are otherwise
 * arbitrary (edges are zero-filled on load and masked on store).
 *
 * Replaces the reference's per-kernel-file plugin symbol
 *     void launch_kernel(const half*, const half*, float*, const GemmConfig&, cudaStream_t)
 *     void launch_kernel(const int8_t*, const int8_t*, int32_t*, const GemmConfig&, cudaStream_t)
 * (src/solver.cu:6-7, src/solver_int8.h:7-8, src/solver_int4.h:5-6); the
 * reference-compatible C++ symbols live in tcgemm_compat.h.
 */
#ifndef TCGEMM_H
#define TCGEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    TCG_SUCCESS = 0,
    TCG_ERR_SHAPE = 1,       /* a dimension breaks the rules above              */
    TCG_ERR_ALIGN = 2,       /* A or B not 16-byte aligned (C not 4-byte)       */
    TCG_ERR_TIMEOUT = 3,     /* a device-side bounded wait gave up (see below)  */
    TCG_ERR_CUDA = 4,        /* a CUDA runtime call failed (tcg_last_cuda_error) */
    TCG_ERR_ARG = 5,         /* bad enum / null pointer                          */
    TCG_ERR_UNSUPPORTED = 6, /* device is not sm_100 (B200/GB200)                */
    TCG_ERR_WORKSPACE = 7    /* workspace too small                              */
} tcg_status;

typedef enum { TCG_ACC_F32 = 0, TCG_ACC_F16 = 1 } tcg_acc;
typedef enum { TCG_B_KN = 0, TCG_B_NK = 1 } tcg_b_layout;
typedef enum { TCG_F8_E4M3 = 0, TCG_F8_E5M2 = 1 } tcg_f8_format;

/* fp16 x fp16 -> fp32 C, fp32 (TCG_ACC_F32) or fp16 (TCG_ACC_F16) accumulation.
 * Replaces fp16 launch_kernel: kernels/fp16_wmma.cu:92-102 (fp32 acc) and
 * kernels/fp16_ptx_fp16acc.cu:190-200 (fp16 acc, fp32 store). */
tcg_status tcg_gemm_f16(const void* A, const void* B, float* C,
                        int M, int N, int K, int batches,
                        tcg_acc acc, tcg_b_layout b_layout, void* stream);

/* int8 x int8 -> int32, exact.  Replaces int8 launch_kernel:
 * kernels/int8_wmma.cu:135-145, kernels/int8_ptx_mma_k32.cu:162-172. */
tcg_status tcg_gemm_s8(const int8_t* A, const int8_t* B, int32_t* C,
                       int M, int N, int K, int batches,
                       tcg_b_layout b_layout, void* stream);

/* int8 GEMM whose epilogue writes the M x N result to every one of C_dst[0..
 * n_dst-1] (1 <= n_dst <= 8): C_dst[0] is local; the others may be peer GPUs'
 * buffers mapped with tcg_ipc_open, reached with NVLink stores from the same
 * epilogue, so an all-gather of row-sharded C overlaps the tensor-core work
 * tile by tile.  The caller orders readers of peer buffers after this launch
 * (e.g. a collective barrier on the same stream).  No counterpart in the
 * reference, which has no multi-GPU path. */
tcg_status tcg_gemm_s8_multi(const int8_t* A, const int8_t* B, int32_t* const* C_dst, int n_dst,
                             int M, int N, int K, tcg_b_layout b_layout, void* stream);

/* Cross-process peer mapping (CUDA IPC) for tcg_gemm_s8_multi destinations.
 * tcg_ipc_handle: 64-byte handle of the allocation holding `ptr`, and ptr's
 * offset in it.  tcg_ipc_open: map another process's allocation into the
 * current device's address space (base of the allocation; add the offset).
 * tcg_ipc_close: unmap a base returned by tcg_ipc_open. */
tcg_status tcg_ipc_handle(const void* ptr, void* handle, size_t* offset);
tcg_status tcg_ipc_open(const void* handle, void** base);
tcg_status tcg_ipc_close(void* base);

/* fp8 x fp8 -> fp32 C with fp32 accumulation (tcgen05 kind::f8f6f4), each
 * operand e4m3 or e5m2 (OCP FP8).  The reference lists FP8 as planned and
 * never built it (README.md:143-146); same layouts and rules as int8. */
tcg_status tcg_gemm_f8(const void* A, const void* B, float* C, int M, int N, int K, int batches,
                       tcg_f8_format a_fmt, tcg_f8_format b_fmt, tcg_b_layout b_layout, void* stream);

/* packed int4 x int4 -> int32, exact; B is always BT (N x K/2 bytes).
 * Replaces int4 launch_kernel: kernels/int4_wmma.cu:148-158,
 * kernels/int4_ptx_mma_k64_x4_x2nontrans_ca.cu:168-178.
 * One kernel: TMA brings the packed rows into shared memory, converter warps
 * widen them to int8 there, and the int8 tensor-core path multiplies them --
 * like the reference's launch_kernel it allocates nothing, and `workspace`
 * may be NULL.  `workspace` (tcg_gemm_s4_workspace_size bytes, 256-byte
 * aligned) is used only by the two-pass form (operands widened into it by a
 * separate kernel, then the int8 GEMM), which the environment variable
 * TCG_S4_PREPASS=1 selects; in that form a NULL workspace is taken from a
 * stream-ordered private memory pool for the duration of the call. */
size_t tcg_gemm_s4_workspace_size(int M, int N, int K, int batches);
tcg_status tcg_gemm_s4(const int8_t* A_packed, const int8_t* BT_packed, int32_t* C,
                       int M, int N, int K, int batches,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Fused dequantisation (int8 / int4): C (fp32) = (float)(A x B) * (scale_a *
 * scale_b), the step the reference performs on the host after the GEMM
 * (src/data_int8.cu:91-95 dequantize, src/main_int8.cu:170-171).  scale_a and
 * scale_b are device pointers to one float each (e.g. written by
 * tcg_quantize_absmax_*); the arithmetic is the reference's, rounding for
 * rounding.  Other arguments as tcg_gemm_s8 / tcg_gemm_s4. */
tcg_status tcg_gemm_s8_dequant(const int8_t* A, const int8_t* B, float* C, int M, int N, int K, int batches,
                               tcg_b_layout b_layout, const float* scale_a, const float* scale_b, void* stream);
tcg_status tcg_gemm_s4_dequant(const int8_t* A_packed, const int8_t* BT_packed, float* C, int M, int N, int K,
                               int batches, const float* scale_a, const float* scale_b, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Per-tensor absmax quantisation on the device, bit-identical to the
 * reference's quantize_absmax (src/data_int8.cu:74-89: codes in [-127,127],
 * scale = absmax / 127) and quantize_absmax_int4 (src/data_int4.cu:104-127:
 * codes in [-7,7] packed two per byte along each row of cols_k values, scale =
 * absmax / 7).  `scale` is a device float that receives the scale.  src must
 * be 16-byte aligned, dst and scale 4-byte aligned. */
tcg_status tcg_quantize_absmax_s8(const float* src, int8_t* dst, size_t n, float* scale, void* stream);
tcg_status tcg_quantize_absmax_s4(const float* src, int8_t* dst_packed, int rows, int cols_k, float* scale,
                                  void* stream);

/* Widen packed int4 to int8 (low nibble first), n_packed bytes -> 2*n_packed.
 * The first pass of tcg_gemm_s4's two-pass form, exposed for reuse. */
tcg_status tcg_unpack_s4(const int8_t* packed, int8_t* out, size_t n_packed, void* stream);

/* No counterpart in the reference.  tcg_gemm_s4 without allocation.
 *
 * Some callers cannot allocate device memory at all: a host application or
 * serving framework that owns the whole device-memory budget and forbids its
 * plugins to allocate, or a latency-critical path that cannot accept the
 * device-wide synchronisation cudaMalloc implies, or code written to the
 * reference's int4 `launch_kernel` contract, which takes no workspace and
 * allocates nothing.  tcg_gemm_s4's two-pass form needs scratch for the
 * widened operands, so for those callers this variant runs that form with
 * its scratch in one fixed device array inside libtcgemm.so,
 * TCG_S4_STATIC_SCRATCH_BYTES large, that every GPU which loads the library
 * holds until the process exits.  (tcg_gemm_s4's default fused kernel
 * allocates nothing either; this entry keeps the two-pass form available to
 * such callers, e.g. as an independent cross-check.)
 *
 * Same operands, result and status codes as tcg_gemm_s4.  The limit is on
 * the scratch need, tcg_gemm_s4_workspace_size(M, N, K, batches) <=
 * TCG_S4_STATIC_SCRATCH_BYTES, i.e. batches*M*K + batches*N*K bytes (the
 * widened A and B, each rounded up to 256 bytes) of at most 32 MiB: 4096 x
 * 4096 x 4096 fits exactly, and so does 8192 x 8192 x 2048.  Larger problems
 * return TCG_ERR_WORKSPACE and launch nothing.  No cudaMalloc/cudaFree or
 * other allocating routine is called.  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture (a failed lookup
 * is retried by the next call).  cudaDeviceReset while the library is loaded
 * is not supported.  All calls share
 * the one array: calls that overlap on the GPU (other streams, other host
 * threads) race on it and must be serialised by the caller.  The array keeps
 * the last call's contents; every call overwrites all of the scratch it reads,
 * so nothing has to start at zero. */
#define TCG_S4_STATIC_SCRATCH_BYTES (32u << 20)
tcg_status tcg_gemm_s4_static(const int8_t* A_packed, const int8_t* BT_packed, int32_t* C,
                              int M, int N, int K, int batches, void* stream);

/* Strided 2-D copy (height rows of width_bytes), host<->device or
 * device<->device, asynchronous on `stream` (cudaMemcpy2DAsync, direction
 * from the pointers).  Used by the host-buffer GEMM pipeline to move C blocks
 * between contiguous device buffers and a row-major host matrix. */
tcg_status tcg_copy_2d_async(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width_bytes,
                             size_t height, void* stream);

/* Page-lock a host range the caller has mapped (for example a POSIX shared
 * memory segment every process of a job maps) so that copies between it and
 * any GPU run as DMA, like pinned memory from cudaHostAlloc
 * (cudaHostRegister, portable to every device).  Used by the multi-process
 * host-buffer GEMM, whose ranks read A and B from, and write C to, one shared
 * host matrix.  tcg_host_unregister undoes it before the range is unmapped. */
tcg_status tcg_host_register(void* ptr, size_t bytes);
tcg_status tcg_host_unregister(void* ptr);

/* Device-side failure word.  Every wait inside the GEMM kernel is bounded
 * (default 2 s, tcg_set_wait_timeout_ns); on expiry the kernel records
 * (code << 32 | detail) here, drains its own copies in flight, frees its
 * tensor memory and returns.  tcg_check_device_error synchronises `stream`,
 * reads the word of the current device, clears it, and returns
 * TCG_ERR_TIMEOUT if it was set (detail in *word when word != NULL). */
tcg_status tcg_check_device_error(void* stream, uint64_t* word);
void tcg_set_wait_timeout_ns(uint64_t ns);

/* Self-test of the failure path: launches a kernel whose bounded waits (the
 * GEMM's own wait code) watch an mbarrier nothing arrives on; after
 * timeout_ns they record the failure word (detail low byte 0xFF) and the
 * kernel returns.  tcg_check_device_error then reports TCG_ERR_TIMEOUT and
 * the device stays usable.  No counterpart in the reference. */
tcg_status tcg_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

/* Tile overrides for tuning: the tile width (0 = automatic; else 64, 128 or
 * 256) and the tile shape (0 = automatic, 1 = single-CTA 128-row tiles,
 * 2 = two-CTA 256-row tiles, 3 = single-CTA 256 x 256 tiles with two
 * accumulators, 4 = two-CTA 512 x 256 tiles, two accumulators per CTA).
 * Shapes a precision cannot run fall back to the nearest valid one. */
void tcg_set_tile_n(int bn);
void tcg_set_cta_pair(int mode);

/* Introspection: last CUDA error code seen, status names, library version,
 * and the tile shape (width, rows) chosen by the most recent launch on this
 * thread. */
int tcg_last_cuda_error(void);
const char* tcg_status_string(tcg_status s);
int tcg_version(void);
int tcg_last_tile_n(void);
int tcg_last_tile_m(void);

#ifdef __cplusplus
}
#endif
#endif /* TCGEMM_H */
