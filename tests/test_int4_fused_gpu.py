"""The fused int4 GEMM: packed operands widened to int8 in shared memory by
the kernel's converter warps (no scratch, no second pass over HBM), checked
bit for bit against the oracle (the reference's cpu_gemm_int4 restated,
src/data_int4.cu:46-61) on every tile shape, ragged M / N / K (a last k-block
partly outside K reads zero-filled packed bytes), batches and multi-wave
problems whose last wave runs as half tiles."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def rand_s4_packed(rng, rows, k, batches=None):
    shape = (rows, k // 2) if batches is None else (batches, rows, k // 2)
    lo = rng.integers(-8, 8, shape, dtype=np.int8)
    hi = rng.integers(-8, 8, shape, dtype=np.int8)
    return ((lo & 0x0F) | (hi << 4)).astype(np.int8)


def T():
    import tensorcoreptx_b200 as t
    return t


# (cta mode, tile width): 1 one-CTA 128-row tiles, 2 two-CTA 256-row tiles,
# 3 one-CTA 256 x 256 (two accumulators), 4 two-CTA 512 x 256
SHAPES = [(1, 64), (1, 128), (1, 256), (2, 128), (2, 256), (3, 0), (4, 0)]


@pytest.mark.parametrize("mode,bn", SHAPES)
@pytest.mark.parametrize("M,N,K", [(640, 768, 512), (300, 200, 160), (513, 129, 4096)])
def test_int4_fused_every_tile_shape(mode, bn, M, N, K):
    t = T()
    rng = np.random.default_rng(M + N + K + 10 * mode + bn)
    A = rand_s4_packed(rng, M, K)
    BT = rand_s4_packed(rng, N, K)
    ref = O.gemm_s4(A, BT, K, threads=8)
    try:
        t.set_cta_pair(mode)
        t.set_tile_n(bn)
        C = t.gemm_int4(_cuda(A), _cuda(BT)).cpu().numpy()
    finally:
        t.set_cta_pair(0)
        t.set_tile_n(0)
    assert np.array_equal(C, ref)


@pytest.mark.parametrize("M,N,K", [(1, 1, 32), (128, 256, 32), (77, 1000, 96), (256, 384, 1056), (129, 65, 224)])
def test_int4_fused_ragged_bit_exact(M, N, K):
    rng = np.random.default_rng(7 * M + N + K)
    A = rand_s4_packed(rng, M, K)
    BT = rand_s4_packed(rng, N, K)
    C = T().gemm_int4(_cuda(A), _cuda(BT)).cpu().numpy()
    assert np.array_equal(C, O.gemm_s4(A, BT, K, threads=8))


def test_int4_fused_batched():
    rng = np.random.default_rng(17)
    A = rand_s4_packed(rng, 200, 256, batches=3)
    BT = rand_s4_packed(rng, 72, 256, batches=3)
    C = T().gemm_int4(_cuda(A), _cuda(BT)).cpu().numpy()
    for b in range(3):
        assert np.array_equal(C[b], O.gemm_s4(A[b], BT[b], 256))


@pytest.mark.parametrize("M,N,K", [(4096, 2560, 256), (2304, 4096, 512), (8192, 8192, 128)])
def test_int4_fused_multi_wave(M, N, K):
    """More tiles than one wave of SM pairs (work items taken over by cluster
    launch control, half tiles in the last wave, K walked backwards on odd
    waves): exact against the int8 GEMM of the widened operands, plus rows
    against the oracle."""
    t = T()
    rng = np.random.default_rng(M ^ N ^ K)
    A = rand_s4_packed(rng, M, K)
    BT = rand_s4_packed(rng, N, K)
    At, Bt = _cuda(A), _cuda(BT)
    C = t.gemm_int4(At, Bt)
    C8 = t.gemm_int8(t.unpack_int4(At), t.unpack_int4(Bt))
    assert torch.equal(C, C8)
    Cn = C.cpu().numpy()
    for r in (0, M // 2, M - 1):
        assert np.array_equal(Cn[r], O.gemm_s4(A[r:r + 1], BT, K)[0])


def test_int4_fused_allocates_nothing_and_ignores_workspace():
    """The fused path needs no scratch: a NULL workspace and a 1-byte one give
    the same exact result."""
    from tensorcoreptx_b200 import _native as nat
    L = nat.lib()
    rng = np.random.default_rng(5)
    M, N, K = 512, 384, 256
    A, BT = rand_s4_packed(rng, M, K), rand_s4_packed(rng, N, K)
    At, Bt = _cuda(A), _cuda(BT)
    ref = O.gemm_s4(A, BT, K, threads=8)
    s = torch.cuda.current_stream().cuda_stream
    tiny = torch.empty(256, dtype=torch.uint8, device=DEV)
    for ws, nbytes in ((None, 0), (tiny.data_ptr(), 1)):
        C = torch.full((M, N), -3, dtype=torch.int32, device=DEV)
        assert L.tcg_gemm_s4(At.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, 1, ws, nbytes, s) == 0
        assert np.array_equal(C.cpu().numpy(), ref)
