"""The size-independent checks bench.py and the large GPU tests rely on
(tensorcoreptx_b200.verify), exercised on the CPU: they accept the oracle's
exact product and reject a product with one planted wrong element."""
import numpy as np
import torch

from oracle import oracle as O
from tensorcoreptx_b200.verify import freivalds_int8, rows_int8


def _case(M=300, N=260, K=512, seed=0):
    rng = np.random.default_rng(seed)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    BT = rng.integers(-128, 128, (N, K), dtype=np.int8)
    C = O.gemm_s8(A, BT, threads=4)
    return torch.from_numpy(A), torch.from_numpy(BT), torch.from_numpy(C)


def test_freivalds_accepts_the_exact_product():
    A, BT, C = _case()
    assert freivalds_int8(A, BT, C, trials=3, chunk=128)


def test_freivalds_rejects_one_planted_error():
    A, BT, C = _case(seed=1)
    for (i, j, d) in [(0, 0, 1), (299, 259, -1), (150, 7, 1 << 20)]:
        Cb = C.clone()
        Cb[i, j] += d
        # two trials miss a single wrong element with probability <= (1/17)^2;
        # seeds fixed, so the outcome is deterministic
        assert not freivalds_int8(A, BT, Cb, trials=2, seed=5, chunk=64)


def test_rows_match_the_oracle():
    A, BT, C = _case(seed=2)
    rows = [0, 1, 298, 299]
    assert torch.equal(rows_int8(A, BT, rows, chunk=100), C[rows])


def test_freivalds_refuses_sizes_beyond_exactness():
    A = torch.zeros(1, 1 << 16, dtype=torch.int8)
    BT = torch.zeros(1 << 21, 1, dtype=torch.int8).expand(1 << 21, 1 << 16)
    try:
        freivalds_int8(A, BT, torch.zeros(1, 1 << 21, dtype=torch.int32))
    except ValueError:
        return
    raise AssertionError("expected a ValueError")
