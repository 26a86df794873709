"""Time one library operation on seeded synthetic inputs (CUDA events).

    python -m tensorcoreptx_b200.opbench gemm_int8 --m 4096 --n 4096 --k 4096
    python -m tensorcoreptx_b200.opbench quantize_int8 --m 8192 --k 8192 --iters 3

Operations: gemm_int8 (B given as BT, N x K), gemm_int8_kn, gemm_int4 (packed
operands), gemm_fp16 (B K x N; --acc fp32|fp16), gemm_fp8 (e4m3, BT),
gemm_int8_dequant, quantize_int8 / quantize_int4 (an M x K fp32 input);
reference points through torch: torch_int_mm, torch_matmul_fp16.
Prints one line: the operation, its shape, the mean time per call after
warm-up and the rate (TOPS / TFLOP/s for GEMMs, GB/s of algorithmic bytes for
quantisation).  Also the workload for profiling a single kernel under ncu.
"""
from __future__ import annotations

import argparse
import time


OPS = ("gemm_int8", "gemm_int8_kn", "gemm_int4", "gemm_fp16", "gemm_fp8", "gemm_int8_dequant",
       "quantize_int8", "quantize_int4", "torch_int_mm", "torch_matmul_fp16")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("op")
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--acc", choices=["fp32", "fp16"], default="fp32")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    if a.op not in OPS:
        raise SystemExit(f"unknown operation {a.op!r}; one of {', '.join(OPS)}")

    import torch
    import tensorcoreptx_b200 as T

    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(0)
    M, N, K = a.m, a.n, a.k

    def s8(r, c):
        return torch.randint(-128, 128, (r, c), generator=g, device=dev, dtype=torch.int8)

    def f16(r, c):
        return (torch.rand(r, c, generator=g, device=dev) * 2 - 1).half()

    gemm_ops = 2.0 * M * N * K
    if a.op == "gemm_int8":
        A, B = s8(M, K), s8(N, K)
        fn, work, unit = (lambda: T.gemm_int8(A, B)), gemm_ops, "TOPS"
    elif a.op == "gemm_int8_kn":
        A, B = s8(M, K), s8(K, N)
        fn, work, unit = (lambda: T.gemm_int8_kn(A, B)), gemm_ops, "TOPS"
    elif a.op == "gemm_int4":
        A, B = s8(M, K // 2), s8(N, K // 2)
        ws = torch.empty(T.int4_workspace_size(M, N, K), dtype=torch.uint8, device=dev)
        fn, work, unit = (lambda: T.gemm_int4(A, B, ws)), gemm_ops, "TOPS"
    elif a.op == "gemm_fp16":
        A, B = f16(M, K), f16(K, N)
        fn, work, unit = (lambda: T.gemm_fp16(A, B, acc=a.acc)), gemm_ops, "TFLOP/s"
    elif a.op == "gemm_fp8":
        A, B = f16(M, K).to(torch.float8_e4m3fn), f16(N, K).to(torch.float8_e4m3fn)
        fn, work, unit = (lambda: T.gemm_fp8(A, B)), gemm_ops, "TFLOP/s"
    elif a.op == "gemm_int8_dequant":
        qa, sa = T.quantize_absmax_int8(torch.randn(M, K, generator=g, device=dev))
        qb, sb = T.quantize_absmax_int8(torch.randn(N, K, generator=g, device=dev))
        fn, work, unit = (lambda: T.gemm_int8_dequant(qa, qb, sa, sb)), gemm_ops, "TOPS"
    elif a.op == "torch_int_mm":  # reference point: torch / cuBLASLt int8 GEMM, same inputs
        A, B = s8(M, K), s8(N, K)
        fn, work, unit = (lambda: torch._int_mm(A, B.t())), gemm_ops, "TOPS"
    elif a.op == "torch_matmul_fp16":  # reference point: torch / cuBLAS fp16 GEMM
        A, B = f16(M, K), f16(K, N)
        fn, work, unit = (lambda: torch.matmul(A, B)), gemm_ops, "TFLOP/s"
    elif a.op in ("quantize_int8", "quantize_int4"):
        X = torch.randn(M, K, generator=g, device=dev)
        q = T.quantize_absmax_int8 if a.op == "quantize_int8" else T.quantize_absmax_int4
        per = 5.0 if a.op == "quantize_int8" else 4.5  # fp32 read once + codes written
        fn, work, unit = (lambda: q(X)), per * M * K, "GB/s"
    else:
        raise SystemExit(f"unknown operation {a.op!r}")

    for _ in range(a.warmup):
        fn()
    torch.cuda.synchronize()
    time.sleep(0.2)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / a.iters
    rate = work / (ms * 1e-3) / (1e9 if unit == "GB/s" else 1e12)
    shape = f"{M} x {K} fp32" if a.op.startswith("quantize") else f"M={M} N={N} K={K}"
    print(f"{a.op} {shape}: {ms * 1e3:.2f} us per call, {rate:.1f} {unit}")
    if T.check_device_error() != 0:
        raise SystemExit("device-side wait expired")


if __name__ == "__main__":
    main()
