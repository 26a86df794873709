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

from tensorcoreptx_b200.dist import (cyclic_row_blocks, gathered_gemm_int8, max_over_ranks, shard_rows,
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
