// ref_kernel_shim.cu -- C entry point around one reference kernel file
// (test and baseline infrastructure, compiled into oracle/_ref/ only).
//
// Each reference kernel file defines the same C++ symbol `launch_kernel`
// (fp16: kernels/fp16_wmma.cu:92-102; int8/int4: kernels/int8_wmma.cu:135-145,
// kernels/int4_ptx_mma_k64_x4_x2nontrans_ca.cu:168-178).  Linking one kernel
// file with this shim into its own shared library lets the bench and the
// tests load several of them side by side (RTLD_LOCAL) and time the
// reference's own GPU code, recompiled for sm_100a, on the same box.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include "include/config.h"

#if defined(REF_SHIM_FP16)
void launch_kernel(const half* A, const half* B, float* C,
                   const GemmConfig& cfg, cudaStream_t stream);
#elif defined(REF_SHIM_INT)
void launch_kernel(const int8_t* A, const int8_t* BT, int32_t* C,
                   const GemmConfig& cfg, cudaStream_t stream);
#else
#error "define REF_SHIM_FP16 or REF_SHIM_INT"
#endif

extern "C" int ref_launch(const void* A, const void* B, void* C,
                          int M, int N, int K, int batches, void* stream)
{
    GemmConfig cfg{M, N, K, batches, 0, 1};
#if defined(REF_SHIM_FP16)
    launch_kernel(static_cast<const half*>(A), static_cast<const half*>(B),
                  static_cast<float*>(C), cfg, static_cast<cudaStream_t>(stream));
#else
    launch_kernel(static_cast<const int8_t*>(A), static_cast<const int8_t*>(B),
                  static_cast<int32_t*>(C), cfg, static_cast<cudaStream_t>(stream));
#endif
    return static_cast<int>(cudaGetLastError());
}
