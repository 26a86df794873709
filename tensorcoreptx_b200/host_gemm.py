"""GEMM on host-resident operands with copy / compute overlap.

The reference copies whole matrices to the device, runs one launch and copies
C back (src/main_int8.cu:113-122).  Over PCIe the copies dominate: at
M = N = K = 32768 (int8) the step moves 2 GiB in and 4 GiB out for ~30 ms of
tensor-core work.  These entry points take pinned host tensors and pipeline
row chunks of C: while chunk i is multiplied on the caller's current stream,
the A rows of chunk i+1 are copied in on one stream and C rows of chunk i-1
copied out on another (B, which every chunk needs in full, goes first).  The
result lands in a pinned host tensor; like the device entry points, the call
is asynchronous with respect to the host.

Every multiply goes through libtcgemm.so (the C ABI); torch only provides the
pinned/device buffers, streams and events.
"""
from __future__ import annotations

import torch

from . import _native as nat

_STREAMS: dict = {}


def _streams(dev: torch.device):
    key = dev.index
    if key not in _STREAMS:
        _STREAMS[key] = (torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev))
    return _STREAMS[key]


def _check(cond: bool, msg: str):
    if not cond:
        raise RuntimeError(msg)


def _check_host(t: torch.Tensor, name: str, dtype):
    _check(t.device.type == "cpu", f"{name} must be a host tensor")
    _check(t.dtype == dtype, f"{name} must be {str(dtype).replace('torch.', '')}")
    _check(t.dim() == 2 and t.is_contiguous(), f"{name} must be 2-D and contiguous")


def _row_chunks(M: int, chunks: int):
    rows = -(-M // max(1, chunks))
    rows = max(256, -(-rows // 256) * 256)  # whole 256-row tiles per chunk
    return [(r0, min(M, r0 + rows)) for r0 in range(0, M, rows)]


def _pipeline(A_h, B_h, C_h, M, launch, chunks, device):
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    cur = torch.cuda.current_stream(dev)
    s_in, s_out = _streams(dev)
    A_d = torch.empty(A_h.shape, dtype=A_h.dtype, device=dev)
    B_d = torch.empty(B_h.shape, dtype=B_h.dtype, device=dev)
    C_d = torch.empty(C_h.shape, dtype=C_h.dtype, device=dev)
    s_in.wait_stream(cur)
    s_out.wait_stream(cur)
    with torch.cuda.stream(s_in):
        B_d.copy_(B_h, non_blocking=True)
    for (r0, r1) in _row_chunks(M, chunks):
        with torch.cuda.stream(s_in):
            A_d[r0:r1].copy_(A_h[r0:r1], non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(s_in)
        cur.wait_event(ready)
        launch(A_d, B_d, C_d, r0, r1, cur)
        done = torch.cuda.Event()
        done.record(cur)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            C_h[r0:r1].copy_(C_d[r0:r1], non_blocking=True)
    cur.wait_stream(s_out)
    # the device buffers were allocated on `cur` and used on the copy streams
    A_d.record_stream(s_in)
    B_d.record_stream(s_in)
    C_d.record_stream(s_out)
    return C_h


def gemm_int8_host(A: torch.Tensor, BT: torch.Tensor, out: torch.Tensor | None = None,
                   chunks: int = 8, device=None) -> torch.Tensor:
    """C[M,N] int32 = A[M,K] int8 x BT[N,K]^T int8, all three in (pinned) host
    memory; the multiply runs on the current CUDA device, overlapped with the
    copies.  Synchronise the current stream before reading C."""
    _check_host(A, "A", torch.int8)
    _check_host(BT, "BT", torch.int8)
    _check(A.size(1) == BT.size(1), "A cols must equal BT cols (both = K)")
    M, K = A.shape
    N = BT.size(0)
    C = out if out is not None else torch.empty((M, N), dtype=torch.int32, pin_memory=True)
    _check_host(C, "out", torch.int32)
    _check(tuple(C.shape) == (M, N), "out must be M x N")

    def launch(A_d, B_d, C_d, r0, r1, stream):
        st = nat.lib().tcg_gemm_s8(A_d.data_ptr() + r0 * K, B_d.data_ptr(), C_d.data_ptr() + r0 * N * 4,
                                   r1 - r0, N, K, 1, nat.TCG_B_NK, stream.cuda_stream)
        nat.check("gemm_int8_host", st)

    return _pipeline(A, BT, C, M, launch, chunks, device)


def gemm_fp16_host(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor | None = None, acc: str = "fp32",
                   chunks: int = 8, device=None) -> torch.Tensor:
    """C[M,N] fp32 = A[M,K] fp16 x B[K,N] fp16 from (pinned) host memory;
    see gemm_int8_host."""
    _check_host(A, "A", torch.float16)
    _check_host(B, "B", torch.float16)
    _check(A.size(1) == B.size(0), "A cols must equal B rows")
    _check(acc in ("fp32", "fp16"), "acc must be 'fp32' or 'fp16'")
    M, K = A.shape
    N = B.size(1)
    C = out if out is not None else torch.empty((M, N), dtype=torch.float32, pin_memory=True)
    _check_host(C, "out", torch.float32)
    _check(tuple(C.shape) == (M, N), "out must be M x N")
    mode = nat.TCG_ACC_F32 if acc == "fp32" else nat.TCG_ACC_F16

    def launch(A_d, B_d, C_d, r0, r1, stream):
        st = nat.lib().tcg_gemm_f16(A_d.data_ptr() + r0 * K * 2, B_d.data_ptr(), C_d.data_ptr() + r0 * N * 4,
                                    r1 - r0, N, K, 1, mode, nat.TCG_B_KN, stream.cuda_stream)
        nat.check("gemm_fp16_host", st)

    return _pipeline(A, B, C, M, launch, chunks, device)
