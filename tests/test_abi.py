"""CPU tests of the drop-in boundary: the C-ABI library loads and exports
every symbol include/tcgemm.h declares, the compat libraries export the
reference's C++ symbols, and host-side validation answers without a GPU."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tensorcoreptx_b200")


def _header_symbols(name):
    text = open(os.path.join(ROOT, "include", name)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tcg_[a-z0-9_]+)\s*\(", text)))


def test_c_abi_exports_every_declared_symbol():
    from tensorcoreptx_b200 import _native
    L = _native.lib()
    declared = _header_symbols("tcgemm.h")
    assert declared, "no declarations parsed"
    for sym in declared:
        assert hasattr(L, sym), sym
    assert set(declared) == set(_native.SIGNATURES), "ctypes table out of sync with header"


@pytest.mark.parametrize("prec,syms", [
    ("f16", ["launch_kernel(__half const*, __half const*, float*, GemmConfig const&, CUstream_st*)",
             "Solver::run(__half const*, __half const*, float*)", "Solver::configure(GemmConfig const&)"]),
    ("s8", ["launch_kernel(signed char const*, signed char const*, int*, GemmConfig const&, CUstream_st*)",
            "SolverInt8::run(signed char const*, signed char const*, int*)"]),
    ("s4", ["launch_kernel(signed char const*, signed char const*, int*, GemmConfig const&, CUstream_st*)",
            "SolverInt4::run(signed char const*, signed char const*, int*)"]),
])
def test_compat_exports_reference_symbols(prec, syms):
    path = os.path.join(PKG, f"libtcgemm_compat_{prec}.so")
    out = subprocess.check_output(["nm", "-DC", "--defined-only", path], text=True)
    for s in syms:
        assert s in out, s
    C.CDLL(path)  # loads (resolves libtcgemm.so through its rpath)


def test_host_validation_without_gpu():
    """Shape/argument rules are checked before any device access."""
    from tensorcoreptx_b200 import _native as n
    L = n.lib()
    # empty problems succeed without touching the device
    assert L.tcg_gemm_s8(None, None, None, 0, 16, 32, 1, n.TCG_B_NK, None) == 0
    assert L.tcg_gemm_f16(None, None, None, 8, 0, 32, 1, 0, 0, None) == 0
    # bad enums / negative sizes / misaligned pointers
    assert L.tcg_gemm_f16(16, 16, 16, 8, 8, 8, 1, 7, 0, None) == 5        # TCG_ERR_ARG
    assert L.tcg_gemm_s8(16, 16, 16, -1, 8, 16, 1, 1, None) == 1          # TCG_ERR_SHAPE
    assert L.tcg_gemm_s8(17, 16, 16, 8, 8, 16, 1, 1, None) == 2           # TCG_ERR_ALIGN (A)
    assert L.tcg_gemm_s8(16, 16, 18, 8, 8, 16, 1, 1, None) == 2           # TCG_ERR_ALIGN (C)
    assert L.tcg_gemm_s8(16, 16, 16, 8, 8, 24, 1, 1, None) == 1           # K % 16
    assert L.tcg_gemm_s8(16, 16, 16, 8, 8, 32, 1, 0, None) == 1           # KN: N % 16
    assert L.tcg_gemm_f16(16, 16, 16, 8, 8, 12, 1, 0, 1, None) == 1       # K % 8
    assert L.tcg_gemm_s4(16, 16, 16, 8, 8, 48, 1, None, 0, None) == 1     # K % 32
    assert L.tcg_gemm_s4_workspace_size(4, 8, 64, 2) == 512 + 1024
    assert L.tcg_status_string(3).decode().startswith("a device-side wait")


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: the Python surface refuses host tensors with the
    reference binding's message."""
    import torch
    import tensorcoreptx_b200 as T
    with pytest.raises(RuntimeError, match="A and B must be CUDA tensors"):
        T.gemm_fp16(torch.zeros(4, 8, dtype=torch.float16), torch.zeros(8, 4, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="A and BT must be CUDA tensors"):
        T.gemm_int8(torch.zeros(4, 16, dtype=torch.int8), torch.zeros(4, 16, dtype=torch.int8))


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from tensorcoreptx_b200 import _native
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(ImportError, match="missing"):
        _native.lib()


def test_host_entry_validation():
    import torch
    import tensorcoreptx_b200 as T
    with pytest.raises(RuntimeError, match="must be int8"):
        T.gemm_int8_host(torch.zeros(4, 16), torch.zeros(4, 16, dtype=torch.int8))
    with pytest.raises(RuntimeError, match="A cols must equal BT cols"):
        T.gemm_int8_host(torch.zeros(4, 16, dtype=torch.int8), torch.zeros(4, 32, dtype=torch.int8))
    from tensorcoreptx_b200.host_gemm import _row_chunks
    assert _row_chunks(1000, 3) == [(0, 512), (512, 1000)]
    assert _row_chunks(100, 8) == [(0, 100)]
    assert _row_chunks(4096, 8) == [(r, r + 512) for r in range(0, 4096, 512)]


def test_host_block_schedule_covers_every_block_once_after_its_operands():
    from tensorcoreptx_b200.host_gemm import _block_schedule
    for mc, nc in ((1, 1), (8, 8), (3, 7), (7, 2)):
        steps = _block_schedule(mc, nc)
        loaded = set()
        mms = []
        for st in steps:
            if st[0] == "mm":
                assert ("a", st[1]) in loaded and ("b", st[2]) in loaded
                mms.append(st[1:])
            else:
                loaded.add(st)
        assert sorted(mms) == [(i, j) for i in range(mc) for j in range(nc)]
        assert loaded == {("a", i) for i in range(mc)} | {("b", j) for j in range(nc)}
        assert steps[:3] == [("a", 0), ("b", 0), ("mm", 0, 0)]


def test_opbench_rejects_unknown_operation_without_a_gpu():
    from tensorcoreptx_b200 import opbench
    with pytest.raises(SystemExit, match="unknown operation"):
        opbench.main(["gemm_int9"])
