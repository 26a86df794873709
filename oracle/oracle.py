"""CPU oracle for the tensor-core GEMM path -- TEST INFRASTRUCTURE ONLY.

This module is the checker.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU legs (``cpu_baseline`` and ``--impl reference``) import it.
The product (``tensorcoreptx_b200``) never imports it and has no CPU fallback.

It wraps two shared libraries:

* ``oracle/liboracle.so`` -- the plain-C restatement of the reference's host
  code (``oracle/tcg_oracle.c``; every function cites the reference
  ``src/data*.cu`` lines it follows);
* ``oracle/libcpu_blocked.so`` -- a cache-blocked, multi-threaded CPU GEMM
  (``oracle/cpu_blocked.c``): the host-core baseline reported beside the GPU
  numbers, exact for integers like the reference's naive loops;
* ``oracle/_ref/libref_data_*.so`` -- the reference's own ``src/data.cu``,
  ``src/data_int8.cu`` and ``src/data_int4.cu`` compiled unchanged from source
  (``make -C oracle ref``).  They pin the restatement and serve as the
  "reference" CPU baseline.  They are optional at run time (absent when the
  reference tree was not available at build time).

Arrays are numpy; fp16 matrices travel as ``uint16`` bit patterns.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_lib = None
_lock = threading.Lock()

_p = C.c_void_p
_i = C.c_int
_l = C.c_long
_f = C.c_float


class AccF32(C.Structure):
    _fields_ = [("max_abs_err", C.c_float), ("rmse", C.c_float),
                ("real_err_pct", C.c_float), ("pass_", C.c_int)]


class AccI32(C.Structure):
    _fields_ = [("max_abs_err", C.c_int32), ("rmse", C.c_float),
                ("max_row", C.c_int), ("max_col", C.c_int),
                ("ref_at_max", C.c_int32), ("out_at_max", C.c_int32),
                ("pass_", C.c_int)]


class AccQuant(C.Structure):
    _fields_ = [("max_abs_err", C.c_float), ("rmse", C.c_float),
                ("real_err_pct", C.c_float), ("snr_db", C.c_float),
                ("pass_", C.c_int)]


def _build_if_missing():
    if not os.path.exists(LIB_PATH):
        import subprocess
        subprocess.check_call(["make", "-s", "-C", HERE, "all"])


def lib():
    global _lib
    with _lock:
        if _lib is None:
            _build_if_missing()
            L = C.CDLL(LIB_PATH)
            sig = {
                "oracle_f32_to_f16": (C.c_uint16, [C.c_float]),
                "oracle_f16_to_f32": (C.c_float, [C.c_uint16]),
                "oracle_generate_fp16": (None, [_p, _p, _i, _i, _i, _i]),
                "oracle_generate_int8": (None, [_p, _p, _i, _i, _i, _i]),
                "oracle_generate_int4_packed": (None, [_p, _p, _i, _i, _i, _i]),
                "oracle_generate_fp32_normal": (None, [_p, _p, _i, _i, _i, _i]),
                "oracle_gemm_f16_f32acc": (None, [_p, _p, _p, _i, _i, _i, _i, _i]),
                "oracle_gemm_f16_f64": (None, [_p, _p, _p, _i, _i, _i, _i, _i, _i]),
                "oracle_gemm_s8": (None, [_p, _p, _p, _i, _i, _i, _i, _i]),
                "oracle_gemm_s8_kn": (None, [_p, _p, _p, _i, _i, _i, _i, _i]),
                "oracle_gemm_s4": (None, [_p, _p, _p, _i, _i, _i, _i, _i]),
                "oracle_gemm_f32": (None, [_p, _p, _p, _i, _i, _i, _i, _i]),
                "oracle_unpack_s4": (None, [_p, _p, _l]),
                "oracle_f8_to_f64": (C.c_double, [C.c_uint8, _i]),
                "oracle_gemm_f8_f64": (None, [_p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _i]),
                "oracle_quantize_absmax_s8": (C.c_float, [_p, _p, _l]),
                "oracle_quantize_absmax_s4": (C.c_float, [_p, _p, _i, _i]),
                "oracle_dequantize": (None, [_p, _p, _l, _f, _f]),
                "oracle_measure_accuracy": (AccF32, [_p, _p, _i, _i, _f]),
                "oracle_measure_accuracy_i32": (AccI32, [_p, _p, _i, _i]),
                "oracle_measure_accuracy_quant": (AccQuant, [_p, _p, _i, _i, _f]),
            }
            for name, (res, args) in sig.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


_blocked = None


def blocked_lib():
    """oracle/libcpu_blocked.so (built on first use like liboracle.so)."""
    global _blocked
    with _lock:
        if _blocked is None:
            path = os.path.join(HERE, "libcpu_blocked.so")
            if not os.path.exists(path):
                import subprocess
                subprocess.check_call(["make", "-s", "-C", HERE, "all"])
            L = C.CDLL(path)
            L.cpu_blocked_gemm_s8.restype = None
            L.cpu_blocked_gemm_s8.argtypes = [_p, _p, _p, _i, _i, _i, _i]
            L.cpu_blocked_gemm_s4.restype = _i
            L.cpu_blocked_gemm_s4.argtypes = [_p, _p, _p, _i, _i, _i, _i]
            L.cpu_blocked_gemm_f16.restype = _i
            L.cpu_blocked_gemm_f16.argtypes = [_p, _p, _p, _i, _i, _i, _i]
            _blocked = L
    return _blocked


def blocked_gemm_s8(A, BT, threads=1):
    """C = A x BT^T (int8 -> int32) with the blocked multi-threaded CPU GEMM."""
    A = np.ascontiguousarray(A, np.int8)
    BT = np.ascontiguousarray(BT, np.int8)
    M, K = A.shape
    N = BT.shape[0]
    Cm = np.empty((M, N), np.int32)
    blocked_lib().cpu_blocked_gemm_s8(_ptr(A), _ptr(BT), _ptr(Cm), M, N, K, threads)
    return Cm


def blocked_gemm_s4(Ap, BTp, K, threads=1):
    """C = A x BT^T for packed int4 operands (K/2 bytes per row)."""
    Ap = np.ascontiguousarray(Ap, np.int8)
    BTp = np.ascontiguousarray(BTp, np.int8)
    M, N = Ap.shape[0], BTp.shape[0]
    Cm = np.empty((M, N), np.int32)
    if blocked_lib().cpu_blocked_gemm_s4(_ptr(Ap), _ptr(BTp), _ptr(Cm), M, N, K, threads) != 0:
        raise MemoryError("cpu_blocked_gemm_s4: scratch allocation failed")
    return Cm


def blocked_gemm_f16(A_bits, B_bits, threads=1):
    """C (fp32) = A x B for fp16 bit patterns (A M x K, B K x N)."""
    A_bits = np.ascontiguousarray(A_bits, np.uint16)
    B_bits = np.ascontiguousarray(B_bits, np.uint16)
    M, K = A_bits.shape
    N = B_bits.shape[1]
    Cm = np.empty((M, N), np.float32)
    if blocked_lib().cpu_blocked_gemm_f16(_ptr(A_bits), _ptr(B_bits), _ptr(Cm), M, N, K, threads) != 0:
        raise MemoryError("cpu_blocked_gemm_f16: scratch allocation failed")
    return Cm


# --------------------------------------------------------------------------
# binary16 helpers
# --------------------------------------------------------------------------

def f16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """IEEE binary16 bit patterns -> float32 (exact)."""
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


# --------------------------------------------------------------------------
# reference-compatible generators (glibc rand after srand(42) / srand(43))
# --------------------------------------------------------------------------

def generate_fp16(M, N, K, batches=1):
    A = np.empty(batches * M * K, np.uint16)
    B = np.empty(batches * K * N, np.uint16)
    lib().oracle_generate_fp16(_ptr(A), _ptr(B), M, N, K, batches)
    return A.reshape(batches, M, K), B.reshape(batches, K, N)


def generate_int8(M, N, K, batches=1):
    A = np.empty(batches * M * K, np.int8)
    BT = np.empty(batches * N * K, np.int8)
    lib().oracle_generate_int8(_ptr(A), _ptr(BT), M, N, K, batches)
    return A.reshape(batches, M, K), BT.reshape(batches, N, K)


def generate_int4_packed(M, N, K, batches=1):
    A = np.empty(batches * M * (K // 2), np.int8)
    BT = np.empty(batches * N * (K // 2), np.int8)
    lib().oracle_generate_int4_packed(_ptr(A), _ptr(BT), M, N, K, batches)
    return A.reshape(batches, M, K // 2), BT.reshape(batches, N, K // 2)


def generate_fp32_normal(M, N, K, batches=1):
    A = np.empty(batches * M * K, np.float32)
    BT = np.empty(batches * N * K, np.float32)
    lib().oracle_generate_fp32_normal(_ptr(A), _ptr(BT), M, N, K, batches)
    return A.reshape(batches, M, K), BT.reshape(batches, N, K)


# --------------------------------------------------------------------------
# GEMMs (one batch).  `rows` restricts the computation to C[row0:row0+rows];
# `threads` splits rows across host threads (ctypes drops the GIL).
# --------------------------------------------------------------------------

def _rows_parallel(fn, M, row0, rows, threads):
    rows = M - row0 if rows is None else rows
    if threads is None:
        threads = 1
    threads = max(1, min(threads, rows)) if rows > 0 else 1
    if threads == 1:
        fn(row0, rows)
        return
    chunk = (rows + threads - 1) // threads
    spans = [(row0 + s, min(chunk, rows - s)) for s in range(0, rows, chunk)]
    with ThreadPoolExecutor(len(spans)) as ex:
        list(ex.map(lambda sp: fn(*sp), spans))


def gemm_f16_f32acc(A, B, row0=0, rows=None, threads=1):
    A = np.ascontiguousarray(A, np.uint16)
    B = np.ascontiguousarray(B, np.uint16)
    M, K = A.shape
    N = B.shape[1]
    Cm = np.zeros((M, N), np.float32)
    _rows_parallel(lambda r0, n: lib().oracle_gemm_f16_f32acc(
        _ptr(A), _ptr(B), _ptr(Cm), M, N, K, r0, n), M, row0, rows, threads)
    return Cm


def gemm_f16_f64(A, B, b_kn=True, row0=0, rows=None, threads=1):
    A = np.ascontiguousarray(A, np.uint16)
    B = np.ascontiguousarray(B, np.uint16)
    M, K = A.shape
    N = B.shape[1] if b_kn else B.shape[0]
    Cm = np.zeros((M, N), np.float64)
    _rows_parallel(lambda r0, n: lib().oracle_gemm_f16_f64(
        _ptr(A), _ptr(B), _ptr(Cm), M, N, K, int(b_kn), r0, n), M, row0, rows, threads)
    return Cm


def gemm_s8(A, BT, row0=0, rows=None, threads=1):
    A = np.ascontiguousarray(A, np.int8)
    BT = np.ascontiguousarray(BT, np.int8)
    M, K = A.shape
    N = BT.shape[0]
    Cm = np.zeros((M, N), np.int32)
    _rows_parallel(lambda r0, n: lib().oracle_gemm_s8(
        _ptr(A), _ptr(BT), _ptr(Cm), M, N, K, r0, n), M, row0, rows, threads)
    return Cm


def gemm_s8_kn(A, B, row0=0, rows=None):
    A = np.ascontiguousarray(A, np.int8)
    B = np.ascontiguousarray(B, np.int8)
    M, K = A.shape
    N = B.shape[1]
    Cm = np.zeros((M, N), np.int32)
    lib().oracle_gemm_s8_kn(_ptr(A), _ptr(B), _ptr(Cm), M, N, K, row0,
                            M - row0 if rows is None else rows)
    return Cm


def gemm_s4(Ap, BTp, K, row0=0, rows=None, threads=1):
    Ap = np.ascontiguousarray(Ap, np.int8)
    BTp = np.ascontiguousarray(BTp, np.int8)
    M = Ap.shape[0]
    N = BTp.shape[0]
    Cm = np.zeros((M, N), np.int32)
    _rows_parallel(lambda r0, n: lib().oracle_gemm_s4(
        _ptr(Ap), _ptr(BTp), _ptr(Cm), M, N, K, r0, n), M, row0, rows, threads)
    return Cm


def gemm_f32(A, BT):
    A = np.ascontiguousarray(A, np.float32)
    BT = np.ascontiguousarray(BT, np.float32)
    M, K = A.shape
    N = BT.shape[0]
    Cm = np.zeros((M, N), np.float32)
    lib().oracle_gemm_f32(_ptr(A), _ptr(BT), _ptr(Cm), M, N, K, 0, M)
    return Cm


def unpack_s4(packed):
    packed = np.ascontiguousarray(packed, np.int8)
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), np.int8)
    lib().oracle_unpack_s4(_ptr(packed), _ptr(out), packed.size)
    return out


# --------------------------------------------------------------------------
# quantisation and metrics
# --------------------------------------------------------------------------

def quantize_absmax_s8(x):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.shape, np.int8)
    s = lib().oracle_quantize_absmax_s8(_ptr(x), _ptr(q), x.size)
    return q, s


def quantize_absmax_s4(x):
    x = np.ascontiguousarray(x, np.float32)
    rows, k = x.shape
    q = np.empty((rows, k // 2), np.int8)
    s = lib().oracle_quantize_absmax_s4(_ptr(x), _ptr(q), rows, k)
    return q, s


def dequantize(c, scale_a, scale_bt):
    c = np.ascontiguousarray(c, np.int32)
    out = np.empty(c.shape, np.float32)
    lib().oracle_dequantize(_ptr(c), _ptr(out), c.size, scale_a, scale_bt)
    return out


def measure_accuracy(ref, out, pass_tol=1e-2):
    ref = np.ascontiguousarray(ref, np.float32)
    out = np.ascontiguousarray(out, np.float32)
    M, N = ref.shape
    return lib().oracle_measure_accuracy(_ptr(ref), _ptr(out), M, N, pass_tol)


def measure_accuracy_i32(ref, out):
    ref = np.ascontiguousarray(ref, np.int32)
    out = np.ascontiguousarray(out, np.int32)
    M, N = ref.shape
    return lib().oracle_measure_accuracy_i32(_ptr(ref), _ptr(out), M, N)


def measure_accuracy_quant(ref, out, pass_tol):
    ref = np.ascontiguousarray(ref, np.float32)
    out = np.ascontiguousarray(out, np.float32)
    M, N = ref.shape
    return lib().oracle_measure_accuracy_quant(_ptr(ref), _ptr(out), M, N, pass_tol)


# --------------------------------------------------------------------------
# fp16 tolerance used throughout: max|dC| <= 1e-2 * sqrt(K) * max|A| * max|B|
# --------------------------------------------------------------------------

def fp16_tolerance(A_bits, B_bits, K):
    a = float(np.abs(f16_bits_to_f32(A_bits)).max()) if A_bits.size else 0.0
    b = float(np.abs(f16_bits_to_f32(B_bits)).max()) if B_bits.size else 0.0
    return 1e-2 * np.sqrt(K) * a * b


# --------------------------------------------------------------------------
# the reference's own host code, compiled unchanged into oracle/_ref/
# --------------------------------------------------------------------------

_ref_libs = {}


def ref_data_lib(which: str):
    """Load oracle/_ref/libref_data_<which>.so (which in fp16|int8|int4) or
    return None when the reference was not available at build time."""
    if which in _ref_libs:
        return _ref_libs[which]
    path = os.path.join(REF_DIR, f"libref_data_{which}.so")
    L = None
    if os.path.exists(path):
        L = C.CDLL(path, mode=os.RTLD_LOCAL | os.RTLD_NOW)
        if which == "int8":
            L.gen = L._Z13generate_int8PaS_iiii
            L.gemm = L._Z13cpu_gemm_int8PKaS0_Piiii
        elif which == "int4":
            L.gen = L._Z20generate_int4_packedPaS_iiii
            L.gemm = L._Z13cpu_gemm_int4PKaS0_Piiii
        else:
            L.gen = L._Z13generate_fp16P6__halfS0_iiii
            L.gemm = L._Z13cpu_gemm_fp16PK6__halfS1_Pfiii
        L.gen.restype = None
        L.gen.argtypes = [_p, _p, _i, _i, _i, _i]
        L.gemm.restype = None
        L.gemm.argtypes = [_p, _p, _p, _i, _i, _i]
    _ref_libs[which] = L
    return L


def ref_gemm_rows(which, A, B, M, N, K, Cout, row0, rows, threads=1):
    """Run the reference's own cpu_gemm_<which> on C rows [row0,row0+rows),
    split over `threads` host threads (each call gets a row slice of A and
    C, which the reference's loop indexes from row 0)."""
    L = ref_data_lib(which)
    if L is None:
        raise RuntimeError("oracle/_ref not built")
    abytes = {"int8": K, "int4": K // 2, "fp16": 2 * K}[which]
    cbytes = 4 * N
    a0 = A.ctypes.data
    c0 = Cout.ctypes.data
    b0 = B.ctypes.data

    def run(r0, n):
        L.gemm(C.c_void_p(a0 + r0 * abytes), C.c_void_p(b0),
               C.c_void_p(c0 + r0 * cbytes), n, N, K)

    _rows_parallel(run, M, row0, rows, threads)


def gemm_f8_f64(A, B, a_fmt=0, b_fmt=0, b_kn=False, row0=0, rows=None, threads=1):
    """fp64 product of fp8 operands given as uint8 codes (fmt 0 = e4m3,
    1 = e5m2); B is N x K (b_kn=False) or K x N."""
    A = np.ascontiguousarray(A, np.uint8)
    B = np.ascontiguousarray(B, np.uint8)
    M, K = A.shape
    N = B.shape[1] if b_kn else B.shape[0]
    Cm = np.zeros((M, N), np.float64)
    _rows_parallel(lambda r0, n: lib().oracle_gemm_f8_f64(
        _ptr(A), _ptr(B), _ptr(Cm), M, N, K, a_fmt, b_fmt, int(b_kn), r0, n), M, row0, rows, threads)
    return Cm
