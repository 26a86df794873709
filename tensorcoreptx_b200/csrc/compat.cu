// compat.cu -- reference-compatible launch_kernel + Solver, one precision per
// build (-DTCG_COMPAT_F16 / -DTCG_COMPAT_S8 / -DTCG_COMPAT_S4), each linked
// against libtcgemm.so.  See include/tcgemm_compat.h for the contract.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "tcgemm.h"
#include "tcgemm_compat.h"

namespace {

// The reference's error behaviour (include/cuda_utils.h:5-12): report, exit(1).
void die_on(tcg_status s, const char* what)
{
    if (s == TCG_SUCCESS) return;
    std::fprintf(stderr, "tcgemm error in %s: %s (cuda error %d)\n", what, tcg_status_string(s),
                 tcg_last_cuda_error());
    std::exit(1);
}

void die_on_cuda(cudaError_t e, const char* what)
{
    if (e == cudaSuccess) return;
    std::fprintf(stderr, "CUDA Error in %s: %s\n", what, cudaGetErrorString(e));
    std::exit(1);
}

// Warm-up loop, then `runs` launches between two events on a private stream;
// returns the average milliseconds per launch (src/solver.cu:11-28).
template <class Launch>
float timed_runs(const GemmConfig& cfg, Launch launch)
{
    cudaStream_t st;
    die_on_cuda(cudaStreamCreate(&st), "cudaStreamCreate");
    for (int i = 0; i < cfg.warmups; ++i) launch(st);
    die_on_cuda(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    cudaEvent_t e0, e1;
    die_on_cuda(cudaEventCreate(&e0), "cudaEventCreate");
    die_on_cuda(cudaEventCreate(&e1), "cudaEventCreate");
    die_on_cuda(cudaEventRecord(e0, st), "cudaEventRecord");
    for (int i = 0; i < cfg.runs; ++i) launch(st);
    die_on_cuda(cudaEventRecord(e1, st), "cudaEventRecord");
    die_on_cuda(cudaEventSynchronize(e1), "cudaEventSynchronize");
    float ms = 0.f;
    die_on_cuda(cudaEventElapsedTime(&ms, e0, e1), "cudaEventElapsedTime");
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    die_on_cuda(cudaStreamDestroy(st), "cudaStreamDestroy");
    return cfg.runs > 0 ? ms / cfg.runs : 0.f;
}

}  // namespace

#if defined(TCG_COMPAT_F16)

static tcg_acc compat_acc()
{
    const char* s = std::getenv("TCG_ACC");
    return (s && std::strcmp(s, "fp16") == 0) ? TCG_ACC_F16 : TCG_ACC_F32;
}

void launch_kernel(const half* A, const half* B, float* C, const GemmConfig& cfg, cudaStream_t stream)
{
    die_on(tcg_gemm_f16(A, B, C, cfg.M, cfg.N, cfg.K, cfg.num_batches, compat_acc(), TCG_B_KN, stream),
           "launch_kernel(fp16)");
}

void Solver::configure(const GemmConfig& cfg) { cfg_ = cfg; }

float Solver::run(const half* d_A, const half* d_B, float* d_C)
{
    return timed_runs(cfg_, [&](cudaStream_t st) { launch_kernel(d_A, d_B, d_C, cfg_, st); });
}

#elif defined(TCG_COMPAT_S8)

void launch_kernel(const int8_t* A, const int8_t* BT, int32_t* C, const GemmConfig& cfg, cudaStream_t stream)
{
    die_on(tcg_gemm_s8(A, BT, C, cfg.M, cfg.N, cfg.K, cfg.num_batches, TCG_B_NK, stream), "launch_kernel(int8)");
}

void SolverInt8::configure(const GemmConfig& cfg) { cfg_ = cfg; }

float SolverInt8::run(const int8_t* d_A, const int8_t* d_BT, int32_t* d_C)
{
    return timed_runs(cfg_, [&](cudaStream_t st) { launch_kernel(d_A, d_BT, d_C, cfg_, st); });
}

#elif defined(TCG_COMPAT_S4)

// The reference's int4 signature has no workspace, and its launch_kernel
// allocates nothing (kernels/int4_wmma.cu:148-158); neither does this one:
// the int4 kernel widens the packed operands in shared memory.
void launch_kernel(const int8_t* A, const int8_t* BT, int32_t* C, const GemmConfig& cfg, cudaStream_t stream)
{
    die_on(tcg_gemm_s4(A, BT, C, cfg.M, cfg.N, cfg.K, cfg.num_batches, nullptr, 0, stream),
           "launch_kernel(int4)");
}

void SolverInt4::configure(const GemmConfig& cfg) { cfg_ = cfg; }

float SolverInt4::run(const int8_t* d_A, const int8_t* d_BT, int32_t* d_C)
{
    return timed_runs(cfg_, [&](cudaStream_t st) { launch_kernel(d_A, d_BT, d_C, cfg_, st); });
}

#else
#error "define one of TCG_COMPAT_F16, TCG_COMPAT_S8, TCG_COMPAT_S4"
#endif
