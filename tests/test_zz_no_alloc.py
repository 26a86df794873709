"""tcg_gemm_s4_static: the int4 GEMM for callers that may not allocate.

Some users of this library cannot let it allocate device memory: a host
framework that owns the GPU's whole memory budget and forbids plugins to
allocate, a latency-critical path that cannot take cudaMalloc's implicit
device synchronisation, or code written to the reference's int4
`launch_kernel`, which has no workspace argument and allocates nothing.
tcg_gemm_s4 needs scratch for the widened operands; tcg_gemm_s4_static keeps
that scratch in one fixed device array inside libtcgemm.so instead.

This file is named to be collected last, so a `-x` run has finished every
other test before it.  It calls the entry point through the C ABI (ctypes on
libtcgemm.so) and checks it, bit for bit, against tcg_gemm_s4 with a
caller-provided workspace, on two different problems in a row (the second
smaller, so stale scratch from the first would show), and, in a fresh child
process, that repeated calls take no device memory.
"""
import ctypes as C
import os
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TCG_ERR_WORKSPACE = 7
STATIC_BYTES = 32 << 20   # TCG_S4_STATIC_SCRATCH_BYTES in include/tcgemm.h


def _lib():
    from tensorcoreptx_b200 import _native
    return _native.lib()


def _packed(g, rows, k):
    return torch.randint(-128, 128, (rows, k // 2), generator=g, device=DEV, dtype=torch.int8)


def _existing(L, A, B, M, N, K, stream):
    need = L.tcg_gemm_s4_workspace_size(M, N, K, 1)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    C_ = torch.empty(M, N, dtype=torch.int32, device=DEV)
    st = L.tcg_gemm_s4(A.data_ptr(), B.data_ptr(), C_.data_ptr(), M, N, K, 1, ws.data_ptr(), need, stream)
    assert st == 0, st
    return C_


def _static(L, A, B, M, N, K, stream):
    C_ = torch.full((M, N), -7, dtype=torch.int32, device=DEV)
    st = L.tcg_gemm_s4_static(A.data_ptr(), B.data_ptr(), C_.data_ptr(), M, N, K, 1, stream)
    assert st == 0, st
    return C_


def test_static_scratch_matches_workspace_path_twice():
    torch.cuda.set_device(0)
    L = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=DEV).manual_seed(2024)
    # call 1 fills the whole 32 MiB array (the 4096^3 benchmark shape) ...
    shapes = [(4096, 4096, 4096), (320, 192, 512)]
    for (M, N, K) in shapes:
        assert L.tcg_gemm_s4_workspace_size(M, N, K, 1) <= STATIC_BYTES
        A = _packed(g, M, K)
        B = _packed(g, N, K)
        got = _static(L, A, B, M, N, K, stream)
        want = _existing(L, A, B, M, N, K, stream)
        torch.cuda.synchronize()
        # ... and call 2, smaller, must not see call 1's leftovers
        assert torch.equal(got, want), (M, N, K)
    assert L.tcg_check_device_error(stream, None) == 0


def test_static_scratch_rejects_oversize_without_launching():
    L = _lib()
    M, N, K = 4096, 4096 + 256, 4096
    assert L.tcg_gemm_s4_workspace_size(M, N, K, 1) > STATIC_BYTES
    A = torch.zeros(M, K // 2, dtype=torch.int8, device=DEV)
    B = torch.zeros(N, K // 2, dtype=torch.int8, device=DEV)
    C_ = torch.full((M, N), 5, dtype=torch.int32, device=DEV)
    st = L.tcg_gemm_s4_static(A.data_ptr(), B.data_ptr(), C_.data_ptr(), M, N, K, 1,
                              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert st == TCG_ERR_WORKSPACE
    assert int(C_[0, 0]) == 5 and int(C_[-1, -1]) == 5


_CHILD = textwrap.dedent("""
    import torch
    from tensorcoreptx_b200 import _native
    L = _native.lib()
    torch.cuda.set_device(0)
    M = N = K = 4096
    need = L.tcg_gemm_s4_workspace_size(M, N, K, 1)
    g = torch.Generator(device="cuda:0").manual_seed(7)
    A = torch.randint(-128, 128, (M, K // 2), generator=g, device="cuda:0", dtype=torch.int8)
    B = torch.randint(-128, 128, (N, K // 2), generator=g, device="cuda:0", dtype=torch.int8)
    C = torch.empty(M, N, dtype=torch.int32, device="cuda:0")
    s = torch.cuda.current_stream().cuda_stream
    # the first call loads the kernels (lazy module loading takes device
    # memory for code) and looks up the array's address
    assert L.tcg_gemm_s4_static(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, 1, s) == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert L.tcg_gemm_s4_static(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, 1, s) == 0
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    # any device allocation of the scratch would take `need` bytes (32 MiB)
    assert free0 - free1 < need, (free0, free1, need)
    print("NOALLOC_OK", free0 - free1)
""")


def test_static_scratch_takes_no_device_memory_in_a_fresh_process():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _CHILD], cwd=root, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "NOALLOC_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
