"""GEMM on host-resident operands with copy / compute overlap.

The reference copies whole matrices to the device, runs one launch and copies
C back (src/main_int8.cu:113-122).  Over PCIe the copies dominate: at
M = N = K = 32768 (int8) the step moves 2 GiB in and 4 GiB out for ~25 ms of
tensor-core work.  These entry points take pinned host tensors and split C
into blocks (row chunks x column chunks): block (i, j) is multiplied on the
caller's current stream once row chunk i of A and column chunk j of B are on
the device, while further operand chunks are copied in on one stream and
finished C blocks copied out (strided, into the row-major host C) on
another.  The result lands in a pinned host tensor; like the device entry
points, the call is asynchronous with respect to the host.

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


def _block_schedule(mc: int, nc: int):
    """Inbound copies and block multiplies in order of readiness.

    Operand chunks go in alternately (A_0, B_0, A_1, B_1, ...); after each one
    every block whose two operand chunks are now on the device is multiplied
    (an "L" of new blocks).  Returns a list of ("a", i), ("b", j) and
    ("mm", i, j) steps.  The number of ready blocks grows with the square of
    the chunks copied in, so the outbound copies of finished blocks -- the
    larger half of the PCIe traffic -- start after one A and one B chunk and
    then never wait for work.
    """
    steps = []
    for s in range(max(mc, nc)):
        if s < mc:
            steps.append(("a", s))
            steps += [("mm", s, j) for j in range(min(s, nc))]
        if s < nc:
            steps.append(("b", s))
            steps += [("mm", i, s) for i in range(min(s + 1, mc))]
    return steps


def _pipeline2d(M, N, blocks, dev, copy_a, copy_b, launch, copy_c):
    """Run C = A x B block by block over three streams: inbound copies on one,
    block multiplies on the caller's current stream (each waits for its two
    operand chunks), outbound copies of finished blocks on the third, in the
    order of _block_schedule."""
    cur = torch.cuda.current_stream(dev)
    s_in, s_out = _streams(dev)
    rows = _row_chunks(M, blocks[0])
    cols = _row_chunks(N, blocks[1])
    s_in.wait_stream(cur)
    s_out.wait_stream(cur)
    ready = {}
    waited = set()
    for step in _block_schedule(len(rows), len(cols)):
        if step[0] in ("a", "b"):
            kind, idx = step
            with torch.cuda.stream(s_in):
                (copy_a if kind == "a" else copy_b)(*(rows if kind == "a" else cols)[idx], s_in)
                ev = torch.cuda.Event()
                ev.record(s_in)
            ready[(kind, idx)] = ev
            continue
        _, i, j = step
        for key in (("a", i), ("b", j)):
            if key not in waited:
                cur.wait_event(ready[key])
                waited.add(key)
        (r0, r1), (c0, c1) = rows[i], cols[j]
        launch(r0, r1, c0, c1, cur)
        done = torch.cuda.Event()
        done.record(cur)
        s_out.wait_event(done)
        copy_c(r0, r1, c0, c1, s_out)
    cur.wait_stream(s_out)


def _blocks_for(M, N, chunks):
    return (max(1, min(chunks, -(-M // 256))), max(1, min(chunks, -(-N // 256))))


def _c_block_offsets(M, N, blocks):
    """Start (elements) of each contiguous device C block, 256-byte aligned."""
    offs, at = {}, 0
    for (r0, r1) in _row_chunks(M, blocks[0]):
        for (c0, c1) in _row_chunks(N, blocks[1]):
            offs[(r0, c0)] = at
            at += -(-((r1 - r0) * (c1 - c0)) // 64) * 64
    return offs, at


def gemm_int8_host(A: torch.Tensor, BT: torch.Tensor, out: torch.Tensor | None = None,
                   chunks: int = 8, device=None, group=None) -> torch.Tensor:
    """C[M,N] int32 = A[M,K] int8 x BT[N,K]^T int8, all three in (pinned) host
    memory; the multiply runs on the current CUDA device in chunks x chunks
    blocks overlapped with the copies.  Synchronise the current stream before
    reading C.

    Row-sharded use (one process per GPU, A and C this rank's rows, BT the
    same on every rank): with ``group`` given (a torch.distributed group of
    more than one rank), every rank copies only its 1/G share of each column
    chunk of BT from host memory and the chunk is all-gathered over the group
    (NCCL; NVLink between the GPUs of one box), so each byte of B crosses PCIe
    once per step instead of once per rank.  Every rank of the group must make
    the same call (same N, K and chunks) in the same order; a rank may have no
    rows (M = 0: it only takes part in gathering B), which lets a job keep the
    rows on the GPUs with the fastest path to host memory."""
    _check_host(A, "A", torch.int8)
    _check_host(BT, "BT", torch.int8)
    _check(A.size(1) == BT.size(1), "A cols must equal BT cols (both = K)")
    M, K = A.shape
    N = BT.size(0)
    C = out if out is not None else torch.empty((M, N), dtype=torch.int32, pin_memory=True)
    _check_host(C, "out", torch.int32)
    _check(tuple(C.shape) == (M, N), "out must be M x N")
    if group is not None:
        # the collectives follow the column chunks: every rank must reach
        # them, also a rank without rows (it still copies its share of B)
        _check(N > 0, "row-sharded use needs columns on every rank")
    if N == 0 or (M == 0 and group is None):
        return C
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    blocks = _blocks_for(M, N, chunks)
    offs, c_elems = _c_block_offsets(M, N, blocks)
    A_d = torch.empty((M, K), dtype=torch.int8, device=dev)
    B_d = torch.empty((N, K), dtype=torch.int8, device=dev)
    C_d = torch.empty(max(1, c_elems), dtype=torch.int32, device=dev)
    L = nat.lib()

    def copy_a(r0, r1, stream):
        A_d[r0:r1].copy_(A[r0:r1], non_blocking=True)

    world = 1
    if group is not None:
        import torch.distributed as dist
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)

    def copy_b(c0, c1, stream):
        if world > 1 and (c1 - c0) % world == 0:
            # this rank's share of the chunk from host memory, the rest from
            # the other ranks (in-place all-gather on this stream's order)
            import torch.distributed as dist
            sh = (c1 - c0) // world
            mine = B_d[c0 + rank * sh:c0 + (rank + 1) * sh]
            mine.copy_(BT[c0 + rank * sh:c0 + (rank + 1) * sh], non_blocking=True)
            dist.all_gather_into_tensor(B_d[c0:c1], mine, group=group)
        else:
            B_d[c0:c1].copy_(BT[c0:c1], non_blocking=True)

    def launch(r0, r1, c0, c1, stream):
        st = L.tcg_gemm_s8(A_d.data_ptr() + r0 * K, B_d.data_ptr() + c0 * K,
                           C_d.data_ptr() + offs[(r0, c0)] * 4, r1 - r0, c1 - c0, K, 1, nat.TCG_B_NK,
                           stream.cuda_stream)
        nat.check("gemm_int8_host", st)

    def copy_c(r0, r1, c0, c1, stream):
        st = L.tcg_copy_2d_async(C.data_ptr() + (r0 * N + c0) * 4, N * 4, C_d.data_ptr() + offs[(r0, c0)] * 4,
                                 (c1 - c0) * 4, (c1 - c0) * 4, r1 - r0, stream.cuda_stream)
        nat.check("gemm_int8_host", st)

    _pipeline2d(M, N, blocks, dev, copy_a, copy_b, launch, copy_c)
    s_in, s_out = _streams(dev)
    A_d.record_stream(s_in)
    B_d.record_stream(s_in)
    C_d.record_stream(s_out)
    return C


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
    if M == 0 or N == 0:
        return C
    mode = nat.TCG_ACC_F32 if acc == "fp32" else nat.TCG_ACC_F16
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    blocks = _blocks_for(M, N, chunks)
    offs, c_elems = _c_block_offsets(M, N, blocks)
    A_d = torch.empty((M, K), dtype=torch.float16, device=dev)
    # B column blocks are stored one after another, each K x cols contiguous
    b_offs, at = {}, 0
    for (c0, c1) in _row_chunks(N, blocks[1]):
        b_offs[c0] = at
        at += -(-(K * (c1 - c0)) // 128) * 128
    B_d = torch.empty(max(1, at), dtype=torch.float16, device=dev)
    C_d = torch.empty(max(1, c_elems), dtype=torch.float32, device=dev)
    L = nat.lib()

    def copy_a(r0, r1, stream):
        A_d[r0:r1].copy_(A[r0:r1], non_blocking=True)

    def copy_b(c0, c1, stream):
        st = L.tcg_copy_2d_async(B_d.data_ptr() + b_offs[c0] * 2, (c1 - c0) * 2, B.data_ptr() + c0 * 2, N * 2,
                                 (c1 - c0) * 2, K, stream.cuda_stream)
        nat.check("gemm_fp16_host", st)

    def launch(r0, r1, c0, c1, stream):
        st = L.tcg_gemm_f16(A_d.data_ptr() + r0 * K * 2, B_d.data_ptr() + b_offs[c0] * 2,
                            C_d.data_ptr() + offs[(r0, c0)] * 4, r1 - r0, c1 - c0, K, 1, mode, nat.TCG_B_KN,
                            stream.cuda_stream)
        nat.check("gemm_fp16_host", st)

    def copy_c(r0, r1, c0, c1, stream):
        st = L.tcg_copy_2d_async(C.data_ptr() + (r0 * N + c0) * 4, N * 4, C_d.data_ptr() + offs[(r0, c0)] * 4,
                                 (c1 - c0) * 4, (c1 - c0) * 4, r1 - r0, stream.cuda_stream)
        nat.check("gemm_fp16_host", st)

    _pipeline2d(M, N, blocks, dev, copy_a, copy_b, launch, copy_c)
    s_in, s_out = _streams(dev)
    A_d.record_stream(s_in)
    B_d.record_stream(s_in)
    C_d.record_stream(s_out)
    return C
