"""Row-sharded GEMM over NCCL on 2 GPUs (skipped with fewer GPUs): every
rank's gathered C -- one all-gather after the GEMM, block-cyclic blocks
gathered while the next multiplies, and the GEMM epilogue's peer stores --
equals the single-GPU product of the full matrices; so does the host-buffer
GEMM of each rank's rows with B copied in halves and all-gathered, also with
A, B and C in host memory shared by the ranks and unequal row shares (one
of them with no rows on rank 0)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from tensorcoreptx_b200.dist import shard_rows, sharded_gemm_int8
    import tensorcoreptx_b200 as T
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        M, N, K = 1024, 768, 512
        g = torch.Generator(device=dev).manual_seed(7)  # identical inputs on every rank
        A = torch.randint(-128, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
        BT = torch.randint(-128, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
        r0, r1 = shard_rows(M, world, rank, align=256)
        C = sharded_gemm_int8(A[r0:r1].contiguous(), BT, gather=True)
        full = T.gemm_int8(A, BT)
        ok = bool(torch.equal(C, full))
        # block-cyclic shards, each block gathered while the next multiplies
        from tensorcoreptx_b200.dist import cyclic_row_blocks, gathered_gemm_int8
        A_cyc = torch.cat([A[b0:b1] for b0, b1 in cyclic_row_blocks(M, world, rank, 4)]).contiguous()
        Cg = gathered_gemm_int8(A_cyc, BT, 4)
        torch.cuda.synchronize()
        ok = ok and bool(torch.equal(Cg, full))
        # the same gather through the GEMM epilogue over peer memory, twice
        from tensorcoreptx_b200.dist import PeerGather
        with PeerGather(M, N, dev) as pg:
            for _ in range(2):
                pg.C.fill_(-1)
                dist.barrier()
                Cp = pg.gemm_int8(A[r0:r1].contiguous(), BT, r0)
                torch.cuda.synchronize()
                ok = ok and bool(torch.equal(Cp, full))
            dist.barrier()
        # host-buffer GEMM of this rank's rows with B shared: each rank copies
        # half of every column chunk of BT from host memory, NCCL gathers it
        A_h = A[r0:r1].cpu().pin_memory()
        BT_h = BT.cpu().pin_memory()
        for chunks in (2, 3):
            C_h = T.gemm_int8_host(A_h, BT_h, chunks=chunks, group=dist.group.WORLD)
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(C_h, full[r0:r1].cpu()))
        # the same with A, B and C in host memory shared by the ranks and
        # unequal row shares (as the end-to-end step balances them): every
        # rank's rows land in the one shared C, which then equals the product
        from tensorcoreptx_b200.dist import SharedHostTensor, balanced_rows
        sh = {k: SharedHostTensor(shape, dt, tag=k) for k, shape, dt in
              (("A", (M, K), torch.int8), ("B", (N, K), torch.int8), ("C", (M, N), torch.int32))}
        if rank == 0:
            sh["A"].tensor.copy_(A.cpu())
            sh["B"].tensor.copy_(BT.cpu())
        dist.barrier()
        # 384 / 640 rows (unequal, not 256-aligned), and all rows on rank 1
        # (rank 0 only takes part in gathering B)
        for rates, act in (([1.0, 3.0], None), ([2.0, 1.0], None), ([1.0, 1.0], [False, True])):
            a0, a1 = balanced_rows(M, rates, 128, active=act)[rank]
            sh["C"].tensor[a0:a1].fill_(-1)
            T.gemm_int8_host(sh["A"].tensor[a0:a1], sh["B"].tensor, out=sh["C"].tensor[a0:a1], chunks=2,
                             group=dist.group.WORLD)
            torch.cuda.synchronize()
            dist.barrier()
            ok = ok and bool(torch.equal(sh["C"].tensor, full.cpu()))
            dist.barrier()
        for v in sh.values():
            v.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_gather_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in res:
        assert ok, (rank, err)
