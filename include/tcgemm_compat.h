// tcgemm_compat.h -- reference-compatible C++ entry points.
//
// A program written against MattJBorowski1991/TensorCorePTX links one of
//   libtcgemm_compat_f16.so  -> fp16 launch_kernel + Solver
//   libtcgemm_compat_s8.so   -> int8 launch_kernel + SolverInt8
//   libtcgemm_compat_s4.so   -> int4 launch_kernel + SolverInt4
// in place of one kernels/*.cu file (+ src/solver*.cu), exactly as the
// reference links one kernel file per binary (CMakeLists.txt:31-57).  The int8
// and int4 launch_kernel share one C++ signature (src/solver_int8.h:7-8,
// src/solver_int4.h:5-6), so they live in different libraries.
//
// Semantics follow the reference: A is M x K row-major; fp16 B is K x N
// row-major and C is fp32; int8/int4 B is passed transposed (BT, N x K); int4
// buffers hold two values per byte along K (low nibble = even k) and K counts
// values, not bytes; batch b is at offset b*M*K, b*K*N, b*M*N; C is
// overwritten; the launch is asynchronous on `stream`.  As in the reference
// (include/cuda_utils.h:5-12), a failure prints a message and exits(1).
// The fp16 library accumulates in fp32, or in fp16 when the environment
// variable TCG_ACC=fp16 is set (the reference's fp16_ptx_fp16acc build).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef TCG_GEMMCONFIG_DEFINED
#define TCG_GEMMCONFIG_DEFINED
// Same members and layout as the reference's GemmConfig (include/config.h:16-20).
struct GemmConfig {
    int M, N, K;
    int num_batches;
    int warmups, runs;
};
#endif

// libtcgemm_compat_f16.so -- replaces kernels/fp16_*.cu launch_kernel
// (e.g. kernels/fp16_wmma.cu:92-102).
void launch_kernel(const half* A, const half* B, float* C, const GemmConfig& cfg, cudaStream_t stream);

// libtcgemm_compat_s8.so (int8) and libtcgemm_compat_s4.so (packed int4):
// replaces kernels/int8_*.cu / kernels/int4_*.cu launch_kernel
// (e.g. kernels/int8_ptx_mma_k32.cu:162-172, kernels/int4_wmma.cu:148-158).
void launch_kernel(const int8_t* A, const int8_t* BT, int32_t* C, const GemmConfig& cfg,
                   cudaStream_t stream);

// src/solver.h:6-13 (libtcgemm_compat_f16.so)
class Solver {
public:
    void configure(const GemmConfig& cfg);
    // Average kernel time in milliseconds over cfg.runs timed launches.
    float run(const half* d_A, const half* d_B, float* d_C);

private:
    GemmConfig cfg_{};
};

// src/solver_int8.h:10-17 (libtcgemm_compat_s8.so)
class SolverInt8 {
public:
    void configure(const GemmConfig& cfg);
    float run(const int8_t* d_A, const int8_t* d_BT, int32_t* d_C);

private:
    GemmConfig cfg_{};
};

// src/solver_int4.h:8-14 (libtcgemm_compat_s4.so)
class SolverInt4 {
public:
    void configure(const GemmConfig& cfg);
    float run(const int8_t* d_A, const int8_t* d_BT, int32_t* d_C);

private:
    GemmConfig cfg_{};
};
