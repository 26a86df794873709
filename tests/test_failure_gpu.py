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
