"""Row-sharded multi-GPU GEMM: one process per GPU over torch.distributed.

The reference has no multi-GPU code; this is the sharded configuration its
benchmark calls for: A is partitioned by rows across the ranks, B is
replicated, and each rank computes its rows of C with the local tensor-core
GEMM.  No collective is on the data path; ``gather=True`` adds an all-gather
of C (NCCL over NVLink on GPUs) so every rank ends with the full C.

Failure behaviour: collectives use the process group's timeout, so a rank
that dies or never joins turns into an error on the others instead of a hang.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_rows(M: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Rows [r0, r1) of an M-row matrix owned by `rank` of `world`.

    Shards are as equal as `align` allows (every boundary but the last is a
    multiple of `align`); earlier ranks get the larger shards.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    units = -(-M // align)
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    return min(M, u0 * align), min(M, u1 * align)


def balanced_rows(M: int, rates, align: int = 256, active=None) -> list[tuple[int, int]]:
    """Split M rows into len(rates) consecutive ranges, range i about
    proportional to rates[i] (rows per second that rank i moves between host
    and device), in whole blocks of `align` rows (the last non-empty range
    ends at M).  Ranks with active[i] False get an empty range; every active
    rank gets at least one block while M has one per active rank."""
    n = len(rates)
    if n < 1:
        raise ValueError("no ranks")
    act = [True] * n if active is None else [bool(x) for x in active]
    if not any(act):
        raise ValueError("no active rank")
    w = [max(float(r), 0.0) if a else 0.0 for r, a in zip(rates, act)]
    if sum(w) <= 0.0:
        w = [1.0 if a else 0.0 for a in act]
    n_act = sum(act)
    units = -(-M // align)
    floor_units = 1 if units >= n_act else 0
    free = units - floor_units * n_act
    tot = sum(w)
    share = [free * x / tot for x in w]
    got = [int(x) for x in share]
    # largest remainders take the blocks left over
    for i in sorted((i for i in range(n) if act[i]), key=lambda i: share[i] - got[i],
                    reverse=True)[:free - sum(got)]:
        got[i] += 1
    out, u = [], 0
    for i in range(n):
        u1 = u + (floor_units + got[i] if act[i] else 0)
        out.append((min(M, u * align), min(M, u1 * align)))
        u = u1
    return out


def rebalance_rows(M: int, split, seconds, align: int = 256, damping: float = 0.5) -> list[tuple[int, int]]:
    """The next split after a step in which rank i took seconds[i] for the
    rows split[i]: each rank's rate (rows per second) sets its share, and
    the new shares are moved only `damping` of the way from the old ones, so
    that ranks coupled by collectives settle instead of oscillating.  Ranks
    without rows stay without rows."""
    rows = [r1 - r0 for r0, r1 in split]
    act = [r > 0 for r in rows]
    rates = [r / max(t, 1e-9) for r, t in zip(rows, seconds)]
    tot_r = sum(rates) or 1.0
    target = [M * x / tot_r for x in rates]
    mixed = [(1.0 - damping) * r + damping * t for r, t in zip(rows, target)]
    return balanced_rows(M, mixed, align, active=act)


def choose_host_rows(M: int, run_step: Callable[[int, int], float], group=None,
                     device: Optional[torch.device] = None, align: int = 256, rounds: int = 3):
    """Pick which ranks of `group` take which rows of an M-row host-buffer
    step, by timing the step itself.  `run_step(r0, r1)` runs one step with
    this rank's rows [r0, r1) and returns its time (any unit); every rank
    calls this function with the same M, align and rounds.

    The ranks' paths to host memory differ and share the host's bandwidth,
    so for each candidate set -- all ranks, then the fastest half and the
    fastest quarter by the rate each reached with all of them -- `rounds`
    damped rounds move rows in proportion to each rank's measured rows per
    time unit (rebalance_rows), and the split whose step ended soonest (the
    better of its last two rounds) is returned with the log of every round:
    (split, [{"rows": [...], "ms": [...]}, ...]).  Ranks outside the chosen
    set get no rows."""
    world = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
    rank = dist.get_rank(group) if world > 1 else 0

    def gathered(t: float) -> list[float]:
        if world == 1:
            return [float(t)]
        mine = torch.tensor([float(t)], dtype=torch.float64, device=device)
        every = torch.empty(world, dtype=torch.float64, device=device)
        dist.all_gather_into_tensor(every, mine, group=group)
        return every.tolist()

    sizes = [world] + [k for k in (world // 2, world // 4) if k >= 1 and k != world]
    rates = None
    best = None
    log = []
    for k in dict.fromkeys(sizes):
        if rates is None:
            act = [True] * world
        else:
            top = sorted(range(world), key=lambda i: (-rates[i], i))[:k]
            act = [i in top for i in range(world)]
        sp = balanced_rows(M, [1.0] * world, align, active=act)
        ends = []
        for r in range(rounds):
            secs = gathered(run_step(*sp[rank]))
            log.append({"rows": [b1 - b0 for b0, b1 in sp], "ms": [round(x, 2) for x in secs]})
            ends.append((max(secs), sp))
            if rates is None and r == rounds - 1:
                rates = [(b1 - b0) / max(t, 1e-9) for (b0, b1), t in zip(sp, secs)]
            sp = rebalance_rows(M, sp, secs, align)
        cand = min(ends[-2:], key=lambda e: e[0])
        if best is None or cand[0] < best[0]:
            best = cand
    return best[1], log


class SharedHostTensor:
    """One host tensor mapped by every rank of a process group (a POSIX
    shared-memory segment), page-locked in each process for DMA.

    Lets the ranks of one node exchange rows of A, B and C through host
    memory: whichever GPU has the fastest path to host memory can read or
    write any rows.  Rank 0 creates the segment under a name drawn for this
    job and removes the name once every rank has mapped it, so nothing stays
    behind in /dev/shm when the job ends.  `pin=False` maps it without
    page-locking (CPU-only use).  Collective: every rank of `group` makes the
    same call.  close() unpins it; the mapping goes with the last reference.
    """

    def __init__(self, shape, dtype: torch.dtype, group=None, tag: str = "buf", pin: bool = True,
                 root: str = "/dev/shm"):
        import os
        import uuid

        rank = dist.get_rank(group)
        self.shape = tuple(int(d) for d in shape)
        numel = 1
        for d in self.shape:
            numel *= d
        self.nbytes = numel * torch.empty((), dtype=dtype).element_size()
        names = [os.path.join(root, f"tcg_{tag}_{uuid.uuid4().hex}") if rank == 0 else None]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(names, src=src, group=group)
        path = names[0]
        if rank == 0:
            with open(path, "wb") as f:
                f.truncate(self.nbytes)
        dist.barrier(group)
        self.tensor = torch.from_file(path, shared=True, size=numel, dtype=dtype).view(self.shape)
        dist.barrier(group)
        if rank == 0:
            os.unlink(path)
        self.pinned = False
        if pin and self.nbytes > 0:
            from . import _native as nat
            nat.check("tcg_host_register", nat.lib().tcg_host_register(self.tensor.data_ptr(), self.nbytes))
            self.pinned = True

    def close(self):
        if self.pinned:
            from . import _native as nat
            nat.check("tcg_host_unregister", nat.lib().tcg_host_unregister(self.tensor.data_ptr()))
            self.pinned = False


def max_over_ranks(x: float, device: Optional[torch.device] = None, group=None) -> float:
    """Maximum of a host scalar over all ranks (identity when not distributed)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64,
                     device=device if device is not None else torch.device("cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def sharded_gemm_int8(A_local: torch.Tensor, BT: torch.Tensor, gather: bool = False,
                      out: Optional[torch.Tensor] = None, group=None,
                      local_gemm: Optional[Callable] = None) -> torch.Tensor:
    """C rows of this rank = A_local x BT^T (int8 -> int32); with gather=True
    return the full C (rows of rank r at the position shard_rows gives them,
    equal shards required) after an all-gather over `group`.

    `local_gemm` defaults to the tensor-core GEMM (gemm_int8).
    """
    if local_gemm is None:
        from .gemm import gemm_int8 as local_gemm
    C_local = local_gemm(A_local, BT)
    if not gather:
        return C_local
    world = dist.get_world_size(group)
    rows = C_local.shape[0]
    if out is None:
        out = torch.empty((rows * world, C_local.shape[1]), dtype=C_local.dtype, device=C_local.device)
    if out.shape[0] != rows * world:
        raise RuntimeError("gather needs equal shards: out must have world x local rows")
    dist.all_gather_into_tensor(out, C_local.contiguous(), group=group)
    return out


def cyclic_row_blocks(M: int, world: int, rank: int, chunks: int) -> list[tuple[int, int]]:
    """Block-cyclic row shards: the M rows are `chunks` groups of `world`
    blocks of M / (chunks * world) rows; `rank` owns block `rank` of every
    group.  Returns its [r0, r1) blocks in order (its local rows, stacked)."""
    if world < 1 or not 0 <= rank < world or chunks < 1:
        raise ValueError("bad rank / world size / chunk count")
    if M % (chunks * world):
        raise ValueError("block-cyclic shards need M divisible by chunks x world")
    ch = M // (chunks * world)
    return [(c * world * ch + rank * ch, c * world * ch + (rank + 1) * ch) for c in range(chunks)]


def gathered_gemm_int8(A_local: torch.Tensor, BT: torch.Tensor, chunks: int, out: Optional[torch.Tensor] = None,
                       group=None, local_gemm_into: Optional[Callable] = None) -> torch.Tensor:
    """Full C = A x BT^T on every rank, the all-gather overlapped with the
    GEMM.  A is sharded block-cyclically (``cyclic_row_blocks``): A_local
    stacks this rank's `chunks` row blocks.  Block c is multiplied straight
    into its rows of the full C, then gathered by an in-place all-gather of
    row group c (contiguous, because every rank's block c sits in it), which
    runs while block c+1 is multiplied.

    `local_gemm_into(A_rows, BT, C_rows)` writes A_rows x BT^T into the
    contiguous int32 view C_rows; it defaults to the tensor-core GEMM on the
    current stream.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    rows, K = A_local.shape
    N = BT.shape[0]
    if rows % chunks:
        raise RuntimeError("A_local rows must split into `chunks` equal blocks")
    ch = rows // chunks
    if out is None:
        out = torch.empty((rows * world, N), dtype=torch.int32, device=A_local.device)
    if out.shape != (rows * world, N) or not out.is_contiguous():
        raise RuntimeError("out must be a contiguous (world x local rows) x N int32 tensor")
    if local_gemm_into is None:
        local_gemm_into = _gemm_int8_into
    works = []
    for c in range(chunks):
        group_rows = out[c * world * ch:(c + 1) * world * ch]
        mine = group_rows[rank * ch:(rank + 1) * ch]
        local_gemm_into(A_local[c * ch:(c + 1) * ch], BT, mine)
        works.append(dist.all_gather_into_tensor(group_rows, mine, group=group, async_op=True))
    for w in works:
        w.wait()
    return out


def _gemm_int8_into(A_rows: torch.Tensor, BT: torch.Tensor, C_rows: torch.Tensor):
    """C_rows = A_rows x BT^T with the tensor-core GEMM on the current stream."""
    from . import _native as nat
    from .gemm import _check, _stream_ptr
    _check(A_rows.is_contiguous() and BT.is_contiguous() and C_rows.is_contiguous(),
           "operands must be contiguous")
    M, K = A_rows.shape
    st = nat.lib().tcg_gemm_s8(A_rows.data_ptr(), BT.data_ptr(), C_rows.data_ptr(), M, BT.shape[0], K, 1,
                               nat.TCG_B_NK, _stream_ptr(A_rows))
    nat.check("gathered_gemm_int8", st)


class PeerGather:
    """All-gather of row-sharded C through the GEMM epilogue.

    Every rank allocates the full M x N int32 C; the buffers are mapped into
    every other rank with CUDA IPC (tcg_ipc_*), and ``gemm_int8`` launches one
    tcgen05 GEMM whose epilogue stores each finished tile of this rank's rows
    into all G buffers over NVLink -- the transfer overlaps the math tile by
    tile instead of following it as a separate NCCL all-gather.  A one-word
    all-reduce on the same stream then orders every rank's later reads after
    all ranks' stores.  ``close()`` (or the context manager) unmaps the peer
    buffers; call it on every rank before destroying the process group.
    """

    def __init__(self, M: int, N: int, device: torch.device, group=None):
        import ctypes as C
        from . import _native as nat
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise RuntimeError("PeerGather supports up to 8 ranks")
        self.M, self.N, self.device = M, N, device
        self.C = torch.empty((M, N), dtype=torch.int32, device=device)
        L = nat.lib()
        handle = (C.c_ubyte * 64)()
        off = C.c_size_t(0)
        nat.check("tcg_ipc_handle", L.tcg_ipc_handle(self.C.data_ptr(), handle, C.byref(off)))
        mine = (bytes(handle), int(off.value))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self._opened = []
        self.ptrs = []
        for r, (h, o) in enumerate(allh):
            if r == self.rank:
                self.ptrs.append(self.C.data_ptr())
                continue
            base = C.c_void_p(0)
            buf = (C.c_ubyte * 64).from_buffer_copy(h)
            nat.check("tcg_ipc_open", L.tcg_ipc_open(buf, C.byref(base)))
            self._opened.append(base.value)
            self.ptrs.append(base.value + o)
        self._flag = torch.zeros(1, dtype=torch.int32, device=device)

    def gemm_int8(self, A_local: torch.Tensor, BT: torch.Tensor, row0: int) -> torch.Tensor:
        """Rows [row0, row0 + A_local.shape[0]) of C = A_local x BT^T, stored
        into every rank's full C; returns this rank's full C (complete once
        every rank has made the same call, in stream order)."""
        import ctypes as C
        from . import _native as nat
        from .gemm import _check, _stream_ptr
        _check(A_local.is_cuda and BT.is_cuda, "A and BT must be CUDA tensors")
        _check(A_local.dtype == torch.int8 and BT.dtype == torch.int8, "A and BT must be int8")
        _check(A_local.is_contiguous() and BT.is_contiguous(), "A and BT must be contiguous")
        rows, K = A_local.shape
        _check(BT.shape == (self.N, K), "BT must be N x K")
        _check(0 <= row0 and row0 + rows <= self.M, "rows out of range")
        # this rank's output first (local), then the peers
        order = [self.rank] + [r for r in range(self.world) if r != self.rank]
        dsts = (C.c_void_p * self.world)(*[self.ptrs[r] + row0 * self.N * 4 for r in order])
        st = nat.lib().tcg_gemm_s8_multi(A_local.data_ptr(), BT.data_ptr(), dsts, self.world, rows, self.N, K,
                                         nat.TCG_B_NK, _stream_ptr(A_local))
        nat.check("PeerGather.gemm_int8", st)
        dist.all_reduce(self._flag, group=self.group)  # every rank's stores precede every later read
        return self.C

    def close(self):
        from . import _native as nat
        torch.cuda.synchronize(self.device)
        for base in self._opened:
            nat.lib().tcg_ipc_close(base)
        self._opened = []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
