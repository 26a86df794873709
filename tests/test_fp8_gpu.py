"""fp8 (e4m3 / e5m2) GEMM on tcgen05 kind::f8f6f4 against the oracle's fp64
product of the same fp8 values, within max|dC| <= 1e-2 sqrt(K) max|A| max|B|."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _rand_f8(g, shape, dt):
    return (torch.randn(shape, generator=g, device=DEV) * 2).to(dt)


@pytest.mark.parametrize("afmt,bfmt", [(torch.float8_e4m3fn, torch.float8_e4m3fn),
                                       (torch.float8_e5m2, torch.float8_e5m2),
                                       (torch.float8_e4m3fn, torch.float8_e5m2)])
@pytest.mark.parametrize("M,N,K,layout", [(256, 256, 256, "nk"), (300, 144, 512, "kn"), (1024, 512, 1024, "nk"),
                                           (3328, 2560, 128, "nk")])
def test_fp8_against_fp64(afmt, bfmt, M, N, K, layout):
    import tensorcoreptx_b200 as T
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    A = _rand_f8(g, (M, K), afmt)
    B = _rand_f8(g, (K, N) if layout == "kn" else (N, K), bfmt)
    C = T.gemm_fp8(A, B, b_layout=layout).cpu().numpy()
    fa = 0 if afmt == torch.float8_e4m3fn else 1
    fb = 0 if bfmt == torch.float8_e4m3fn else 1
    Au = A.view(torch.uint8).cpu().numpy()
    Bu = B.view(torch.uint8).cpu().numpy()
    ref = O.gemm_f8_f64(Au, Bu, fa, fb, b_kn=(layout == "kn"), threads=8)
    amax = float(A.float().abs().max())
    bmax = float(B.float().abs().max())
    tol = 1e-2 * np.sqrt(K) * amax * bmax
    err = float(np.abs(C - ref).max())
    assert err <= tol, (err, tol)
    # and far tighter in practice: fp32 accumulation of exact products
    assert err <= 1e-5 * np.sqrt(K) * amax * bmax * 16
