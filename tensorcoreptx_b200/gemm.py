"""Python surface of the GEMM library: the reference's binding functions.

``gemm_fp16(A, B)`` and ``gemm_int8(A, BT)`` keep the names, argument
meaning, checks and error messages of the reference's PyTorch extensions
(bindings/bindings_fp16.cpp:17-37, bindings/bindings_int8.cpp:16-34): checks
raise ``RuntimeError`` as ``TORCH_CHECK`` does, C is a new tensor on the
inputs' device, and the launch is asynchronous on the current stream.
``gemm_int4`` adds the int4 entry the reference never bound (its int4 path
only had the executable, src/main_int4.cu).  All three also accept 3-D
(batched) inputs, the reference's ``num_batches`` (kernels/fp16_wmma.cu:14-18).

Every call goes through libtcgemm.so (the C ABI in include/tcgemm.h); there
is no CPU or library fallback.
"""
from __future__ import annotations

import torch

from . import _native as nat


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_ptr(t: torch.Tensor) -> int:
    """The current CUDA stream of t's device, as a raw handle."""
    if _raw_stream is not None:
        return _raw_stream(t.get_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def _check(cond: bool, msg: str):
    if not cond:
        raise RuntimeError(msg)


def _dims(A, B, b_kn: bool):
    """(batches, M, N, K) for 2-D or matching 3-D operands."""
    _check(A.dim() == B.dim() and A.dim() in (2, 3), "A and B must be 2-D")
    if A.dim() == 3:
        _check(A.size(0) == B.size(0), "A and B must have the same batch count")
    batches = A.size(0) if A.dim() == 3 else 1
    M, K = A.size(-2), A.size(-1)
    N = B.size(-1) if b_kn else B.size(-2)
    return batches, M, N, K


def _out(A, M, N, batches, dtype):
    shape = (batches, M, N) if A.dim() == 3 else (M, N)
    return torch.empty(shape, device=A.device, dtype=dtype)


def gemm_fp16(A: torch.Tensor, B: torch.Tensor, acc: str = "fp32") -> torch.Tensor:
    """C[M,N] fp32 = A[M,K] fp16 x B[K,N] fp16.

    acc="fp32" (fp32 accumulation, the reference's fp16_wmma) or "fp16"
    (fp16 accumulation, the reference's fp16_ptx_fp16acc; C is still fp32).
    """
    _check(A.is_cuda and B.is_cuda, "A and B must be CUDA tensors")
    _check(A.dtype == torch.float16, "A must be fp16")
    _check(B.dtype == torch.float16, "B must be fp16")
    batches, M, N, K = _dims(A, B, b_kn=True)
    _check(K == B.size(-2), "A cols must equal B rows")
    _check(A.is_contiguous() and B.is_contiguous(), "A and B must be contiguous")
    _check(acc in ("fp32", "fp16"), "acc must be 'fp32' or 'fp16'")
    C = _out(A, M, N, batches, torch.float32)
    st = nat.lib().tcg_gemm_f16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, batches,
                                nat.TCG_ACC_F32 if acc == "fp32" else nat.TCG_ACC_F16,
                                nat.TCG_B_KN, _stream_ptr(A))
    nat.check("gemm_fp16", st)
    return C


def gemm_fp16_nk(A: torch.Tensor, BT: torch.Tensor, acc: str = "fp32") -> torch.Tensor:
    """As gemm_fp16 with B given transposed (BT[N,K], K contiguous)."""
    _check(A.is_cuda and BT.is_cuda, "A and BT must be CUDA tensors")
    _check(A.dtype == torch.float16 and BT.dtype == torch.float16, "A and BT must be fp16")
    batches, M, N, K = _dims(A, BT, b_kn=False)
    _check(K == BT.size(-1), "A cols must equal BT cols (both = K)")
    _check(A.is_contiguous() and BT.is_contiguous(), "A and BT must be contiguous")
    _check(acc in ("fp32", "fp16"), "acc must be 'fp32' or 'fp16'")
    C = _out(A, M, N, batches, torch.float32)
    st = nat.lib().tcg_gemm_f16(A.data_ptr(), BT.data_ptr(), C.data_ptr(), M, N, K, batches,
                                nat.TCG_ACC_F32 if acc == "fp32" else nat.TCG_ACC_F16,
                                nat.TCG_B_NK, _stream_ptr(A))
    nat.check("gemm_fp16_nk", st)
    return C


def gemm_int8(A: torch.Tensor, BT: torch.Tensor) -> torch.Tensor:
    """C[M,N] int32 = A[M,K] int8 x BT[N,K]^T int8 (B passed transposed)."""
    _check(A.is_cuda and BT.is_cuda, "A and BT must be CUDA tensors")
    _check(A.dtype == torch.int8, "A must be int8")
    _check(BT.dtype == torch.int8, "BT must be int8")
    batches, M, N, K = _dims(A, BT, b_kn=False)
    _check(K == BT.size(-1), "A cols must equal BT cols (both = K)")
    _check(A.is_contiguous() and BT.is_contiguous(), "A and BT must be contiguous")
    C = _out(A, M, N, batches, torch.int32)
    st = nat.lib().tcg_gemm_s8(A.data_ptr(), BT.data_ptr(), C.data_ptr(), M, N, K, batches,
                               nat.TCG_B_NK, _stream_ptr(A))
    nat.check("gemm_int8", st)
    return C


def gemm_int8_kn(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """C[M,N] int32 = A[M,K] int8 x B[K,N] int8 (B row-major, N contiguous)."""
    _check(A.is_cuda and B.is_cuda, "A and B must be CUDA tensors")
    _check(A.dtype == torch.int8 and B.dtype == torch.int8, "A and B must be int8")
    batches, M, N, K = _dims(A, B, b_kn=True)
    _check(K == B.size(-2), "A cols must equal B rows")
    _check(A.is_contiguous() and B.is_contiguous(), "A and B must be contiguous")
    C = _out(A, M, N, batches, torch.int32)
    st = nat.lib().tcg_gemm_s8(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, batches,
                               nat.TCG_B_KN, _stream_ptr(A))
    nat.check("gemm_int8_kn", st)
    return C


def gemm_int4(A_packed: torch.Tensor, BT_packed: torch.Tensor,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """C[M,N] int32 = A[M,K] int4 x BT[N,K]^T int4, both packed two per byte
    along K (low nibble = even k), i.e. int8 tensors of shape [M, K/2] and
    [N, K/2].  The kernel widens the packed operands in shared memory and
    needs no scratch; `workspace` (>= int4_workspace_size bytes) is only used
    by the two-pass form (TCG_S4_PREPASS=1)."""
    _check(A_packed.is_cuda and BT_packed.is_cuda, "A and BT must be CUDA tensors")
    _check(A_packed.dtype == torch.int8, "A must be int8 (packed int4)")
    _check(BT_packed.dtype == torch.int8, "BT must be int8 (packed int4)")
    batches, M, N, Kh = _dims(A_packed, BT_packed, b_kn=False)
    _check(Kh == BT_packed.size(-1), "A cols must equal BT cols (both = K/2)")
    _check(A_packed.is_contiguous() and BT_packed.is_contiguous(), "A and BT must be contiguous")
    K = 2 * Kh
    ws_ptr, ws_bytes = None, 0
    if workspace is not None:
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    C = _out(A_packed, M, N, batches, torch.int32)
    st = nat.lib().tcg_gemm_s4(A_packed.data_ptr(), BT_packed.data_ptr(), C.data_ptr(), M, N, K,
                               batches, ws_ptr, ws_bytes, _stream_ptr(A_packed))
    nat.check("gemm_int4", st)
    return C


def int4_workspace_size(M: int, N: int, K: int, batches: int = 1) -> int:
    return int(nat.lib().tcg_gemm_s4_workspace_size(M, N, K, batches))


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """Widen packed int4 (int8 tensor, two values per byte, low nibble first)
    to one int8 per value; the last dimension doubles."""
    _check(packed.is_cuda and packed.dtype == torch.int8 and packed.is_contiguous(),
           "packed must be a contiguous CUDA int8 tensor")
    out = torch.empty(packed.shape[:-1] + (2 * packed.shape[-1],), dtype=torch.int8,
                      device=packed.device)
    st = nat.lib().tcg_unpack_s4(packed.data_ptr(), out.data_ptr(), packed.numel(),
                                 _stream_ptr(packed))
    nat.check("unpack_int4", st)
    return out


def check_device_error(stream: torch.cuda.Stream | None = None) -> int:
    """Synchronise `stream` and raise TcgError(TCG_ERR_TIMEOUT) if a kernel on
    this device recorded a bounded-wait expiry; returns the failure word."""
    import ctypes
    s = stream if stream is not None else torch.cuda.current_stream()
    w = ctypes.c_uint64(0)
    st = nat.lib().tcg_check_device_error(s.cuda_stream, ctypes.byref(w))
    nat.check("check_device_error", st)
    return int(w.value)


def set_tile_n(bn: int) -> None:
    """Force the tile width (64, 128, 256); 0 restores automatic choice."""
    nat.lib().tcg_set_tile_n(int(bn))


def set_cta_pair(mode: int) -> None:
    """Force the CTA shape: 0 automatic, 1 single-CTA 128-row tiles, 2 two-CTA
    (cta_group::2) 256-row tiles, 3 single-CTA 256 x 256 tiles, 4 two-CTA
    512 x 256 tiles."""
    nat.lib().tcg_set_cta_pair(int(mode))


def last_tile_n() -> int:
    return int(nat.lib().tcg_last_tile_n())


def last_tile_m() -> int:
    """Rows of C per tile in the most recent launch: 128 (single CTA) or 256 (pair)."""
    return int(nat.lib().tcg_last_tile_m())


# ------------------------------------------------------------- quantisation --

def quantize_absmax_int8(x: torch.Tensor):
    """Per-tensor absmax quantisation on the device: returns (codes int8 with
    x's shape, scale as a 1-element float32 device tensor), bit-identical to
    the reference's quantize_absmax (scale = max|x| / 127, codes rounded half
    away from zero and clamped to [-127, 127])."""
    _check(x.is_cuda and x.dtype == torch.float32 and x.is_contiguous(),
           "x must be a contiguous CUDA float32 tensor")
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    st = nat.lib().tcg_quantize_absmax_s8(x.data_ptr(), q.data_ptr(), x.numel(), scale.data_ptr(),
                                          _stream_ptr(x))
    nat.check("quantize_absmax_int8", st)
    return q, scale


def quantize_absmax_int4(x: torch.Tensor):
    """As quantize_absmax_int8 with scale = max|x| / 7 and codes in [-7, 7]
    packed two per byte along the last dimension (low nibble = even index),
    the reference's quantize_absmax_int4: x [rows, k] -> codes [rows, k/2]."""
    _check(x.is_cuda and x.dtype == torch.float32 and x.is_contiguous() and x.dim() == 2,
           "x must be a contiguous 2-D CUDA float32 tensor")
    rows, k = x.shape
    _check(k % 2 == 0, "x must have an even number of columns")
    q = torch.empty((rows, k // 2), dtype=torch.int8, device=x.device)
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    st = nat.lib().tcg_quantize_absmax_s4(x.data_ptr(), q.data_ptr(), rows, k, scale.data_ptr(), _stream_ptr(x))
    nat.check("quantize_absmax_int4", st)
    return q, scale


def gemm_int8_dequant(A: torch.Tensor, BT: torch.Tensor, scale_a: torch.Tensor,
                      scale_b: torch.Tensor) -> torch.Tensor:
    """C[M,N] fp32 = (A[M,K] int8 x BT[N,K]^T) * (scale_a * scale_b), the
    dequantisation fused into the GEMM epilogue; scales are 1-element float32
    CUDA tensors (e.g. from quantize_absmax_int8)."""
    _check(A.is_cuda and BT.is_cuda, "A and BT must be CUDA tensors")
    _check(A.dtype == torch.int8 and BT.dtype == torch.int8, "A and BT must be int8")
    _check(scale_a.is_cuda and scale_b.is_cuda and scale_a.dtype == torch.float32 and
           scale_b.dtype == torch.float32, "scales must be float32 CUDA tensors")
    batches, M, N, K = _dims(A, BT, b_kn=False)
    _check(K == BT.size(-1), "A cols must equal BT cols (both = K)")
    _check(A.is_contiguous() and BT.is_contiguous(), "A and BT must be contiguous")
    C = _out(A, M, N, batches, torch.float32)
    st = nat.lib().tcg_gemm_s8_dequant(A.data_ptr(), BT.data_ptr(), C.data_ptr(), M, N, K, batches,
                                       nat.TCG_B_NK, scale_a.data_ptr(), scale_b.data_ptr(), _stream_ptr(A))
    nat.check("gemm_int8_dequant", st)
    return C


def gemm_int4_dequant(A_packed: torch.Tensor, BT_packed: torch.Tensor, scale_a: torch.Tensor,
                      scale_b: torch.Tensor) -> torch.Tensor:
    """As gemm_int8_dequant for packed int4 operands [M, K/2] and [N, K/2]."""
    _check(A_packed.is_cuda and BT_packed.is_cuda, "A and BT must be CUDA tensors")
    _check(A_packed.dtype == torch.int8 and BT_packed.dtype == torch.int8, "A and BT must be int8 (packed int4)")
    _check(scale_a.is_cuda and scale_b.is_cuda and scale_a.dtype == torch.float32 and
           scale_b.dtype == torch.float32, "scales must be float32 CUDA tensors")
    batches, M, N, Kh = _dims(A_packed, BT_packed, b_kn=False)
    _check(Kh == BT_packed.size(-1), "A cols must equal BT cols (both = K/2)")
    _check(A_packed.is_contiguous() and BT_packed.is_contiguous(), "A and BT must be contiguous")
    K = 2 * Kh
    C = _out(A_packed, M, N, batches, torch.float32)
    st = nat.lib().tcg_gemm_s4_dequant(A_packed.data_ptr(), BT_packed.data_ptr(), C.data_ptr(), M, N, K,
                                       batches, scale_a.data_ptr(), scale_b.data_ptr(), None, 0,
                                       _stream_ptr(A_packed))
    nat.check("gemm_int4_dequant", st)
    return C


# ----------------------------------------------------------------------- fp8 --

_F8_FORMATS = {torch.float8_e4m3fn: 0, torch.float8_e5m2: 1}


def gemm_fp8(A: torch.Tensor, B: torch.Tensor, b_layout: str = "nk") -> torch.Tensor:
    """C[M,N] fp32 = A[M,K] fp8 x B fp8 with fp32 accumulation on tcgen05
    (kind::f8f6f4).  Operands are torch.float8_e4m3fn or torch.float8_e5m2
    (formats may differ); B is [N,K] (b_layout="nk", K contiguous) or [K,N]
    ("kn")."""
    _check(A.is_cuda and B.is_cuda, "A and B must be CUDA tensors")
    _check(A.dtype in _F8_FORMATS and B.dtype in _F8_FORMATS, "A and B must be float8_e4m3fn or float8_e5m2")
    _check(b_layout in ("nk", "kn"), "b_layout must be 'nk' or 'kn'")
    b_kn = b_layout == "kn"
    batches, M, N, K = _dims(A, B, b_kn=b_kn)
    _check(K == (B.size(-2) if b_kn else B.size(-1)), "A cols must equal K of B")
    _check(A.is_contiguous() and B.is_contiguous(), "A and B must be contiguous")
    C = _out(A, M, N, batches, torch.float32)
    st = nat.lib().tcg_gemm_f8(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, batches,
                               _F8_FORMATS[A.dtype], _F8_FORMATS[B.dtype],
                               nat.TCG_B_KN if b_kn else nat.TCG_B_NK, _stream_ptr(A))
    nat.check("gemm_fp8", st)
    return C
