"""Multi-rank host logic of the row-sharded GEMM, run as gloo ranks on CPU.

The tensor-core GEMM needs a GPU, so here the per-rank multiply is injected
(an exact numpy int64 product, test-only); what is under test is the
partitioning, the all-gather assembly, the max-over-ranks reduction and the
failure behaviour (a rank that leaves turns into an error, not a hang).
"""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tensorcoreptx_b200.dist import (SharedHostTensor, balanced_rows, choose_host_rows, cyclic_row_blocks,
                                     gathered_gemm_int8, max_over_ranks, rebalance_rows, shard_rows,
                                     sharded_gemm_int8)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=60):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _cpu_gemm(A, BT):
    return torch.from_numpy((A.numpy().astype(np.int64) @ BT.numpy().astype(np.int64).T).astype(np.int32))


def _worker_gather(rank, world, port, M, N, K, q):
    try:
        _init(rank, world, port)
        rng = np.random.default_rng(0)  # same full inputs on every rank
        A = torch.from_numpy(rng.integers(-128, 128, (M, K), dtype=np.int8))
        BT = torch.from_numpy(rng.integers(-128, 128, (N, K), dtype=np.int8))
        r0, r1 = shard_rows(M, world, rank)
        C = sharded_gemm_int8(A[r0:r1].contiguous(), BT, gather=True, local_gemm=_cpu_gemm)
        ok = bool(torch.equal(C, _cpu_gemm(A, BT)))
        mx = max_over_ranks(float(rank) * 1.5 + 1.0)
        dist.destroy_process_group()
        q.put((rank, ok, mx))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


def test_shard_rows_partition():
    for M in (0, 1, 7, 256, 1000, 32768):
        for world in (1, 2, 3, 4, 8):
            for align in (1, 256):
                spans = [shard_rows(M, world, r, align) for r in range(world)]
                assert spans[0][0] == 0 and spans[-1][1] == M
                for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                    assert a1 == b0 and a0 <= a1
                    assert a1 % align == 0 or a1 == M
    assert [shard_rows(32768, 8, r) for r in range(8)] == [(r * 4096, (r + 1) * 4096) for r in range(8)]
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def test_cyclic_row_blocks_partition():
    for world in (1, 2, 3, 8):
        for chunks in (1, 2, 4):
            M = world * chunks * 16
            blocks = sorted(b for r in range(world) for b in cyclic_row_blocks(M, world, r, chunks))
            assert blocks[0][0] == 0 and blocks[-1][1] == M
            for (a0, a1), (b0, b1) in zip(blocks, blocks[1:]):
                assert a1 == b0 and a1 - a0 == M // (world * chunks)
    assert cyclic_row_blocks(32, 2, 1, 2) == [(8, 16), (24, 32)]
    with pytest.raises(ValueError):
        cyclic_row_blocks(30, 2, 0, 4)


def _cpu_gemm_into(A_rows, BT, C_rows):
    C_rows.copy_(_cpu_gemm(A_rows, BT))


def _worker_overlap(rank, world, port, M, N, K, chunks, q):
    try:
        _init(rank, world, port)
        rng = np.random.default_rng(1)  # same full inputs on every rank
        A = torch.from_numpy(rng.integers(-128, 128, (M, K), dtype=np.int8))
        BT = torch.from_numpy(rng.integers(-128, 128, (N, K), dtype=np.int8))
        A_local = torch.cat([A[r0:r1] for r0, r1 in cyclic_row_blocks(M, world, rank, chunks)]).contiguous()
        C = gathered_gemm_int8(A_local, BT, chunks, local_gemm_into=_cpu_gemm_into)
        ok = bool(torch.equal(C, _cpu_gemm(A, BT)))
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("world,chunks", [(2, 4), (3, 2)])
def test_overlapped_gather_assembles_full_c(world, chunks):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    M, N, K = world * chunks * 8, 40, 32
    procs = [ctx.Process(target=_worker_overlap, args=(r, world, port, M, N, K, chunks, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in sorted(results):
        assert ok, (rank, err)


@pytest.mark.parametrize("world", [2])
def test_sharded_gemm_gather_and_max_over_ranks(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    M, N, K = 64, 48, 32
    procs = [ctx.Process(target=_worker_gather, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, mx in sorted(results):
        assert ok, (rank, mx)
        assert mx == pytest.approx((world - 1) * 1.5 + 1.0)


def _worker_leaver(rank, world, port, q):
    """Rank 1 leaves between steps; rank 0's next collective must fail within
    the process-group timeout instead of hanging."""
    _init(rank, world, port, timeout_s=5)
    t = torch.ones(4)
    dist.all_reduce(t)  # step 1: both ranks
    if rank == 1:
        q.put((1, "left", 0.0))
        q.close()
        q.join_thread()  # flush the message before leaving
        os._exit(0)  # leaves without finalising
    t0 = time.time()
    try:
        dist.all_reduce(t)  # step 2: peer is gone
        q.put((0, "no error", time.time() - t0))
    except Exception as e:
        q.put((0, type(e).__name__, time.time() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_leaving_becomes_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (what, dt)) for r, what, dt in (q.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():  # pragma: no cover
            p.kill()
    what, dt = results[0]
    assert what != "no error", "collective with a departed rank returned normally"
    assert dt < 60, dt


# ------------------------------------------ host-bandwidth-balanced rows --

def _check_split(split, M, n, align):
    assert len(split) == n
    assert split[0][0] == 0 and max(r1 for _, r1 in split) == M
    for (a0, a1), (b0, b1) in zip(split, split[1:]):
        assert a1 == b0
    for r0, r1 in split:
        assert r1 >= r0
        assert r0 % align == 0 or r0 == M
    if -(-M // align) >= n:
        assert all(r1 > r0 for r0, r1 in split)


def test_balanced_rows_partition_and_proportion():
    for M in (0, 1, 300, 2048, 32768, 32768 + 100):
        for rates in ([1.0], [1, 1], [1, 3], [5, 1, 1, 1], [0, 0, 1], [1] * 8, [18, 18, 18, 18, 44, 44, 44, 44]):
            split = balanced_rows(M, rates, 256)
            _check_split(split, M, len(rates), 256)
    # proportional within one block
    split = balanced_rows(32768, [18, 18, 18, 18, 44, 44, 44, 44], 256)
    rows = [r1 - r0 for r0, r1 in split]
    assert sum(rows) == 32768
    for r, w in zip(rows, [18] * 4 + [44] * 4):
        assert abs(r - 32768 * w / 248) <= 256 + 1e-9
    # equal rates: equal rows
    assert [r1 - r0 for r0, r1 in balanced_rows(32768, [2.0] * 8)] == [4096] * 8
    # inactive ranks get empty ranges, the others share all rows
    act = [False, True, False, True, True, False, False, True]
    split = balanced_rows(32768, [1.0] * 8, 256, active=act)
    assert [r1 - r0 for r0, r1 in split] == [0, 8192, 0, 8192, 8192, 0, 0, 8192]
    assert split[0] == (0, 0) and split[1] == (0, 8192) and split[2] == (8192, 8192)
    nxt = rebalance_rows(32768, split, [1.0, 2.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0])
    assert [r1 - r0 > 0 for r0, r1 in nxt] == act  # inactive stay inactive
    assert nxt[1][1] - nxt[1][0] < 8192  # the slow active rank gives rows away


def test_rebalance_rows_settles_on_rate_shares():
    """A model of ranks whose seconds per row differ 3:1: repeated
    rebalancing converges to the split that equalises their times."""
    M, n = 32768, 4
    cost = [3.0, 3.0, 1.0, 1.0]  # seconds per row (arbitrary units)
    split = balanced_rows(M, [1] * n)
    for _ in range(12):
        secs = [(r1 - r0) * c for (r0, r1), c in zip(split, cost)]
        split = rebalance_rows(M, split, secs)
        _check_split(split, M, n, 256)
    secs = [(r1 - r0) * c for (r0, r1), c in zip(split, cost)]
    assert max(secs) / min(secs) < 1.1


def _worker_shared(rank, world, port, q):
    try:
        _init(rank, world, port)
        sh = SharedHostTensor((world * 4, 8), torch.int32, tag="test", pin=False)
        sh.tensor[rank * 4:(rank + 1) * 4] = rank + 1  # each rank writes its rows
        dist.barrier()
        want = torch.arange(1, world + 1, dtype=torch.int32).repeat_interleave(4)[:, None].expand(world * 4, 8)
        ok = bool(torch.equal(sh.tensor, want))  # every rank sees every rank's rows
        sh.close()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


def test_shared_host_tensor_is_one_buffer_for_all_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    before = set(os.listdir("/dev/shm"))
    procs = [ctx.Process(target=_worker_shared, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in sorted(results):
        assert ok, (rank, err)
    # the segment's name was removed once every rank had mapped it
    assert not [f for f in set(os.listdir("/dev/shm")) - before if f.startswith("tcg_test_")]


def _worker_choose(rank, world, port, q):
    try:
        _init(rank, world, port)
        base = [1.0, 1.0, 3.0, 3.0]  # rows per time unit alone: ranks 0, 1 slow

        def fake_step(r0, r1):
            # a host whose total rate is 5, or 3 while a slow rank copies too,
            # shared in proportion to the active ranks' own rates
            rows = torch.tensor([r1 - r0], dtype=torch.int64)
            every = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(every, rows)
            act = [int(t.item()) > 0 for t in every]
            cap = 3.0 if (act[0] or act[1]) else 5.0
            tot = sum(b for b, a in zip(base, act) if a)
            rate = base[rank] * min(1.0, cap / tot)
            return (r1 - r0) / rate if r1 > r0 else 0.1

        split, log = choose_host_rows(32768, fake_step, align=256, rounds=3)
        rows = [b - a for a, b in split]
        dist.destroy_process_group()
        q.put((rank, rows, len(log)))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), 0))


def test_choose_host_rows_keeps_the_fastest_set():
    """With all four ranks the host moves 3 row units per time unit; with only
    the two fast ranks it moves 5: the search must hand every row to ranks 2
    and 3, equally, and every rank must return the same split."""
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_choose, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    splits = {tuple(rows) if isinstance(rows, list) else rows for _, rows, _ in results}
    assert len(splits) == 1, results
    rows = list(next(iter(splits)))
    assert rows == [0, 0, 16384, 16384], rows
    assert all(n == 9 for _, _, n in results)  # 3 sets x 3 rounds
