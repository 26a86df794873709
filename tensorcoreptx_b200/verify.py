"""Size-independent checks of an int8 GEMM result on the device.

At the full benchmark sizes (M = N = K = 32768: a 4 GiB C) no CPU GEMM can
recompute C in seconds, so the product is checked by properties that are
exact for integers:

* Freivalds' check: ``C x == A (B^T x)`` for random integer vectors x, in
  float64 on the GPU.  With |a|, |b| <= 128, |x| <= 8 and N * K <= 2^36 every
  partial sum is an integer below 2^53 (|C x| and |A (B^T x)| are at most
  N * K * 2^17), so float64 is exact in any summation
  order and a wrong element is caught with probability >= 1 - 1/17 per trial
  (x drawn from 17 values);
* whole rows recomputed in float64 on the GPU (``A[i] . BT[j]`` for every j),
  exact for the same reason.

Both run with torch's float64 kernels, independently of the tensor-core GEMM
being checked.
"""
from __future__ import annotations

import torch


def freivalds_int8(A: torch.Tensor, BT: torch.Tensor, C: torch.Tensor, trials: int = 2, seed: int = 0,
                   chunk: int = 2048) -> bool:
    """True when C == A x BT^T (A M x K int8, BT N x K int8, C M x N int32,
    all on one CUDA device) passes `trials` Freivalds rounds."""
    dev = C.device
    M, K = A.shape
    N = BT.shape[0]
    if N * K > (1 << 36):
        raise ValueError("float64 exactness needs N * K <= 2^36")
    g = torch.Generator(device=dev).manual_seed(seed)
    X = torch.randint(-8, 9, (N, trials), generator=g, device=dev).to(torch.float64)
    y = torch.zeros(K, trials, dtype=torch.float64, device=dev)
    for j0 in range(0, N, chunk):
        y += BT[j0:j0 + chunk].to(torch.float64).t() @ X[j0:j0 + chunk]
    ok = True
    for i0 in range(0, M, chunk):
        lhs = C[i0:i0 + chunk].to(torch.float64) @ X
        rhs = A[i0:i0 + chunk].to(torch.float64) @ y
        ok = ok and bool(torch.equal(lhs, rhs))
    return ok


def rows_int8(A: torch.Tensor, BT: torch.Tensor, rows, chunk: int = 4096) -> torch.Tensor:
    """Rows `rows` of A x BT^T recomputed exactly in float64 (returned as
    int32)."""
    idx = torch.as_tensor(list(rows), device=A.device, dtype=torch.long)
    Ar = A.index_select(0, idx).to(torch.float64)
    N = BT.shape[0]
    out = torch.empty(len(idx), N, dtype=torch.float64, device=A.device)
    for j0 in range(0, N, chunk):
        out[:, j0:j0 + chunk] = Ar @ BT[j0:j0 + chunk].to(torch.float64).t()
    return out.to(torch.int32)
