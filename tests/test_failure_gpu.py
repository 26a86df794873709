"""Failure detection on the GPU without a fault: a bounded wait on an
mbarrier that nothing arrives on must give up, record the failure word, and
leave the context usable (the next GEMM is correct)."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_expiry_is_reported_and_context_survives():
    from tensorcoreptx_b200 import _native as nat
    import tensorcoreptx_b200 as T
    from oracle import oracle as O
    L = nat.lib()
    stream = torch.cuda.current_stream().cuda_stream
    assert L.tcg_check_device_error(stream, None) == 0
    assert L.tcg_selftest_wait_timeout(50_000_000, stream) == 0  # 50 ms
    w = C.c_uint64(0)
    assert L.tcg_check_device_error(stream, C.byref(w)) == nat.TCG_ERR_TIMEOUT
    assert (w.value >> 32) == 1 and (w.value & 0xFF) in (0xFF, 0xFE)
    # the word was cleared, and the device still computes correctly
    assert L.tcg_check_device_error(stream, None) == 0
    rng = np.random.default_rng(3)
    A = rng.integers(-128, 128, (256, 128), dtype=np.int8)
    BT = rng.integers(-128, 128, (192, 128), dtype=np.int8)
    Cm = T.gemm_int8(torch.from_numpy(A).cuda(), torch.from_numpy(BT).cuda()).cpu().numpy()
    assert np.array_equal(Cm, O.gemm_s8(A, BT))
    assert T.check_device_error() == 0


@pytest.mark.parametrize("n,cta_mode", [(512, 0), (4096, 0), (4096, 1), (4096, 2)])
def test_gemm_wait_expiry_aborts_cleanly(n, cta_mode):
    """The GEMM kernel's own abort path.  With a 2 us wait limit the waits of
    a live GEMM run out (the epilogue alone waits ~10-20 us for its first
    accumulator); the kernel records TCG_ERR_TIMEOUT, waits (bounded) for its
    own TMA copies, MMAs and launch-control response, frees its tensor memory
    and returns.  The context stays usable: with the default limit restored
    the same GEMM is exact.  cta_mode: 0 automatic (at 4096^3 two-CTA 512 x
    256 tiles under cluster launch control), 1 one-CTA tiles, 2 two-CTA tiles."""
    from tensorcoreptx_b200 import _native as nat
    import tensorcoreptx_b200 as T
    from tensorcoreptx_b200.verify import freivalds_int8
    L = nat.lib()
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(n + cta_mode)
    A = torch.randint(-128, 128, (n, n), generator=g, device="cuda", dtype=torch.int8)
    BT = torch.randint(-128, 128, (n, n), generator=g, device="cuda", dtype=torch.int8)
    torch.cuda.synchronize()
    assert L.tcg_check_device_error(stream, None) == 0
    w = C.c_uint64(0)
    T.set_cta_pair(cta_mode)
    try:
        L.tcg_set_wait_timeout_ns(2000)
        T.gemm_int8(A, BT)
        st = L.tcg_check_device_error(stream, C.byref(w))
    finally:
        L.tcg_set_wait_timeout_ns(0)  # back to the default limit
        T.set_cta_pair(0)
    assert st in (0, nat.TCG_ERR_TIMEOUT), st
    if st == nat.TCG_ERR_TIMEOUT:
        assert (w.value >> 32) == 1
    torch.cuda.synchronize()  # no CUDA error: the kernel returned
    assert L.tcg_check_device_error(stream, None) == 0
    T.set_cta_pair(cta_mode)
    try:
        Cm = T.gemm_int8(A, BT)
    finally:
        T.set_cta_pair(0)
    assert T.check_device_error() == 0
    assert freivalds_int8(A, BT, Cm)


@pytest.mark.parametrize("cta_mode", [0, 1])
def test_int4_gemm_wait_expiry_aborts_cleanly(cta_mode):
    """The same for the fused int4 kernel, whose converter warps wait on the
    packed staging ring and on the int8 ring's release: with a 2 us limit the
    kernel reports TCG_ERR_TIMEOUT (or finishes), returns, and the next call
    with the default limit is exact."""
    from tensorcoreptx_b200 import _native as nat
    import tensorcoreptx_b200 as T
    L = nat.lib()
    stream = torch.cuda.current_stream().cuda_stream
    n = 4096
    g = torch.Generator(device="cuda").manual_seed(41 + cta_mode)
    Ap = torch.randint(-128, 128, (n, n // 2), generator=g, device="cuda", dtype=torch.int8)
    Bp = torch.randint(-128, 128, (n, n // 2), generator=g, device="cuda", dtype=torch.int8)
    torch.cuda.synchronize()
    assert L.tcg_check_device_error(stream, None) == 0
    T.set_cta_pair(cta_mode)
    try:
        L.tcg_set_wait_timeout_ns(2000)
        T.gemm_int4(Ap, Bp)
        st = L.tcg_check_device_error(stream, None)
    finally:
        L.tcg_set_wait_timeout_ns(0)
        T.set_cta_pair(0)
    assert st in (0, nat.TCG_ERR_TIMEOUT), st
    torch.cuda.synchronize()
    assert L.tcg_check_device_error(stream, None) == 0
    C4 = T.gemm_int4(Ap, Bp)
    C8 = T.gemm_int8(T.unpack_int4(Ap), T.unpack_int4(Bp))
    assert T.check_device_error() == 0
    assert torch.equal(C4, C8)
