"""ctypes binding of libtcgemm.so (the C ABI in include/tcgemm.h).

The library is built in-tree (``python -m tensorcoreptx_b200.build``).  There
is no fallback: if the shared library is missing or fails to load, every op
raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtcgemm.so")

TCG_SUCCESS = 0
TCG_ERR_TIMEOUT = 3
TCG_ACC_F32, TCG_ACC_F16 = 0, 1
TCG_B_KN, TCG_B_NK = 0, 1

STATUS_NAMES = {0: "TCG_SUCCESS", 1: "TCG_ERR_SHAPE", 2: "TCG_ERR_ALIGN", 3: "TCG_ERR_TIMEOUT",
                4: "TCG_ERR_CUDA", 5: "TCG_ERR_ARG", 6: "TCG_ERR_UNSUPPORTED",
                7: "TCG_ERR_WORKSPACE"}

# Every symbol include/tcgemm.h declares, with its ctypes signature.
_p, _i, _sz = C.c_void_p, C.c_int, C.c_size_t
SIGNATURES = {
    "tcg_gemm_f16": (C.c_int, [_p, _p, _p, _i, _i, _i, _i, _i, _i, _p]),
    "tcg_gemm_s8": (C.c_int, [_p, _p, _p, _i, _i, _i, _i, _i, _p]),
    "tcg_gemm_f8": (C.c_int, [_p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _p]),
    "tcg_gemm_s8_multi": (C.c_int, [_p, _p, _p, _i, _i, _i, _i, _i, _p]),
    "tcg_ipc_handle": (C.c_int, [_p, _p, C.POINTER(C.c_size_t)]),
    "tcg_ipc_open": (C.c_int, [_p, C.POINTER(C.c_void_p)]),
    "tcg_ipc_close": (C.c_int, [_p]),
    "tcg_gemm_s4_workspace_size": (_sz, [_i, _i, _i, _i]),
    "tcg_gemm_s4": (C.c_int, [_p, _p, _p, _i, _i, _i, _i, _p, _sz, _p]),
    "tcg_unpack_s4": (C.c_int, [_p, _p, _sz, _p]),
    "tcg_gemm_s8_dequant": (C.c_int, [_p, _p, _p, _i, _i, _i, _i, _i, _p, _p, _p]),
    "tcg_gemm_s4_dequant": (C.c_int, [_p, _p, _p, _i, _i, _i, _i, _p, _p, _p, _sz, _p]),
    "tcg_quantize_absmax_s8": (C.c_int, [_p, _p, _sz, _p, _p]),
    "tcg_quantize_absmax_s4": (C.c_int, [_p, _p, _i, _i, _p, _p]),
    "tcg_gemm_s4_static": (C.c_int, [_p, _p, _p, _i, _i, _i, _i, _p]),
    "tcg_copy_2d_async": (C.c_int, [_p, _sz, _p, _sz, _sz, _sz, _p]),
    "tcg_host_register": (C.c_int, [_p, _sz]),
    "tcg_host_unregister": (C.c_int, [_p]),
    "tcg_check_device_error": (C.c_int, [_p, C.POINTER(C.c_uint64)]),
    "tcg_set_wait_timeout_ns": (None, [C.c_uint64]),
    "tcg_selftest_wait_timeout": (C.c_int, [C.c_uint64, _p]),
    "tcg_set_tile_n": (None, [_i]),
    "tcg_set_cta_pair": (None, [_i]),
    "tcg_last_cuda_error": (C.c_int, []),
    "tcg_status_string": (C.c_char_p, [_i]),
    "tcg_version": (C.c_int, []),
    "tcg_last_tile_n": (C.c_int, []),
    "tcg_last_tile_m": (C.c_int, []),
}

_lib = None
_lock = threading.Lock()


class TcgError(RuntimeError):
    def __init__(self, fn: str, status: int):
        self.status = status
        msg = f"{fn}: {STATUS_NAMES.get(status, status)}"
        try:
            msg += f" ({lib().tcg_status_string(status).decode()})"
            if status == 4:
                msg += f", cuda error {lib().tcg_last_cuda_error()}"
        except Exception:  # pragma: no cover - message decoration only
            pass
        super().__init__(msg)


def lib():
    """Load libtcgemm.so once; raise ImportError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m tensorcoreptx_b200.build`")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(fn: str, status: int):
    if status != TCG_SUCCESS:
        raise TcgError(fn, status)
