#!/usr/bin/env python
"""Benchmark of the tensor-core GEMM path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the sharded int8 GEMM, M = N = K = 32768 in total, int8 uniform
[-128, 127] from a seed, int32 accumulation and output.  A is row-partitioned
across the ranks (M/G rows each), B is replicated, each rank computes its
M/G x N slice of C (no data-path collective in the headline step).  The total
problem is fixed, so scaling is "strong"; at one GPU this is the full 32768^3
problem on one B200.

Inputs: row block b (256 rows) of A and of BT (N x K) is drawn with
torch.randint(-128, 128) from a CPU generator seeded from (matrix, b), so
every rank, and the reference arm, reproduce exactly the rows they need.

A "step" is one GEMM of each rank's slice.  ``value`` is whole-job TOPS with
inputs resident in HBM (2 GiB of operands, larger than L2, so no flush is
needed); ``e2e`` is the same metric through the public host-buffer API
(``gemm_int8_host``): the step's rows of A and B come from pinned host memory
(with more than one GPU each rank copies 1/G of B and the ranks all-gather it
over NVLink) and the rows of C go back, all inside the timed region.  With
more than one GPU, A, B and C are one host matrix each, shared by the ranks,
and the rows of the end-to-end step go to the set of ranks (all, or the
fastest half or quarter) that moved them fastest in calibration steps, split
by each rank's measured throughput (``e2e.rows_per_rank``,
``e2e.balance_rounds``); ranks without rows only help gather B.  Its
bound, ``e2e.copy_floor_ms``, is the same bytes copied with no GEMM (both
directions at once, every rank at once).  Device time is measured with CUDA
events on the launching stream, max over ranks.

After the timed regions (never inside them) the run checks what it timed:
every rank's whole C slice by Freivalds' check and four rows recomputed in
float64 on the GPU, the end-to-end C (against the resident C at one GPU,
each rank's end-to-end rows by Freivalds' check with more), and, at one GPU,
the rows of the CPU-baseline sample against the reference's own
cpu_gemm_int8 -- the ``parity`` object of the line.  At one GPU the line also
carries the reported baselines: the reference's cpu_gemm_int8 and a blocked
multi-threaded CPU GEMM on the host cores, and the reference's GPU kernels
recompiled for sm_100a, each timed on this box.  With more than one GPU the
gathered steps (C all-gathered by the GEMM epilogue's NVLink stores, and by
NCCL) are timed and checked as extras.

``--impl reference`` times the reference's own CPU GEMM (src/data_int8.cu
cpu_gemm_int8, compiled unchanged into oracle/_ref/) on a bounded row sample
of the same workload and the same inputs with all host threads; only rank 0
runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GEMM TFLOPS(fp16)/TOPS(int8,int4) per B200 + % dense tensor peak; 8-GPU agg"
SIZE = 32768
SEED_A, SEED_B = 1234, 999
BLOCK_ROWS = 256


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--size", type=int, default=SIZE, help="M = N = K of the whole problem")
    ap.add_argument("--gather", choices=["none", "nccl", "p2p"], default="none",
                    help="all-gather C in the headline step: NCCL after the GEMM, or peer stores from "
                         "the GEMM epilogue (p2p); the gathered steps are also timed as extras at N > 1")
    ap.add_argument("--no-extras", action="store_true", help="skip the per-config extras")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=8.0,
                    help="target wall time of one CPU-baseline sample")
    return ap.parse_args()


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def workload_config(size, world, gather="none"):
    """The `config` object both arms print (identical for the same run)."""
    return {
        "workload": f"int8 GEMM M=N=K={size}, A row-sharded over {world} GPU(s), B replicated, int32 C"
                    + {"none": "", "nccl": ", C all-gathered (NCCL, block-cyclic rows, 4 blocks each "
                                           "gathered while the next multiplies)",
                       "p2p": ", C all-gathered by the GEMM epilogue over NVLink peer stores"}[gather],
        "per_rank": f"{size // world}x{size}x{size}",
        "values": f"int8 uniform [-128,127]; row block b of A / BT from torch CPU generator seed "
                  f"{SEED_A}*1000003+b / {SEED_B}*1000003+b",
        "l2": "inputs (2 GiB) larger than L2; no flush",
        "parallelism": f"rows{world}",
    }


def gen_rows(seed, r0, r1, cols, threads, out=None):
    """Rows [r0, r1) of the seeded int8 matrix with `cols` columns (a CPU
    tensor).  Row block b is torch.randint(-128, 128) from a CPU generator
    seeded seed * 1000003 + b, so any rows can be reproduced alone."""
    import torch
    n = r1 - r0
    if out is None:
        out = torch.empty((n, cols), dtype=torch.int8)
    b0, b1 = r0 // BLOCK_ROWS, (r1 + BLOCK_ROWS - 1) // BLOCK_ROWS

    def one(b):
        g = torch.Generator().manual_seed(seed * 1000003 + b)
        blk = torch.randint(-128, 128, (BLOCK_ROWS, cols), generator=g, dtype=torch.int8)
        lo, hi = max(r0, b * BLOCK_ROWS), min(r1, (b + 1) * BLOCK_ROWS)
        out[lo - r0:hi - r0] = blk[lo - b * BLOCK_ROWS:hi - b * BLOCK_ROWS]

    with ThreadPoolExecutor(max(1, threads)) as ex:
        list(ex.map(one, range(b0, b1)))
    return out


# ---------------------------------------------------------------- clocks ----

class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 50 ms, each
    sample tagged with the bench phase it fell in ("kernel" = the resident
    timed loop, "e2e" = the end-to-end loop, None = neither)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = gpu_indices
        self.rows = []
        self.proc = None
        self.t = None
        self.active = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", ",".join(str(g) for g in self.gpus)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 9:
                self.rows.append((time.time(), self.active, parts))

    def mark(self, phase):
        self.active = phase

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:  # pragma: no cover
                self.proc.kill()
        if self.t is not None:
            self.t.join(timeout=5)

    def summary(self, phase="kernel"):
        rows = [r for r in self.rows if r[1] == phase]
        window = phase
        if not rows:
            rows = self.rows
            window = "whole run"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"],
                    "samples": 0}
        sm = [float(r[2][1]) for r in rows if r[2][1].replace(".", "").isdigit()]
        mx = [float(r[2][2]) for r in rows if r[2][2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[2][5 + i] == "Active"})
        pw = [float(r[2][3]) for r in rows if r[2][3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_mhz_min": min(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "power_w_max": max(pw) if pw else None, "samples": len(rows), "window": window}




# -------------------------------------------- reference CPU GEMM (sample) ----

def sample_rows(total, n):
    """The CPU sample's rows of a `total`-row slice: the first n/2 and the last
    n - n/2 rows (the slice's edges, where a shard or tile boundary error
    would show)."""
    n = max(2, min(n, total))
    first = n // 2
    return list(range(first)) + list(range(total - (n - first), total))


def cpu_reference_rows(A_rows, BT, threads):
    """The reference's own cpu_gemm_int8 (oracle/_ref) -- or, when the
    reference was not available at build time, the oracle's restatement --
    on the given rows of A (numpy int8, contiguous) against all of BT.
    Returns (C rows, seconds, kind)."""
    import numpy as np
    from oracle import oracle as O

    rows, K = A_rows.shape
    N = BT.shape[0]
    Cs = np.zeros((rows, N), np.int32)
    t0 = time.perf_counter()
    if O.ref_data_lib("int8") is not None:
        O.ref_gemm_rows("int8", A_rows, BT, rows, N, K, Cs, 0, rows, threads=threads)
        kind = "reference"
    else:
        Cs[:] = O.gemm_s8(A_rows, BT, threads=threads)
        kind = "port"
    return Cs, time.perf_counter() - t0, kind


def cpu_sample_count(A_rows_fn, BT, threads, target_s):
    """Rows per sample so one sample takes about target_s seconds (calibrated
    on one row per thread)."""
    _, t, _ = cpu_reference_rows(A_rows_fn(sample_rows(threads * 64, threads)), BT, threads)
    rounds = max(1, int(target_s / max(t, 1e-3)))
    return threads * rounds


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    import numpy as np
    size = args.size
    threads = host_threads()
    BT = gen_rows(SEED_B, 0, size, size, threads).numpy()

    def a_rows(idx):
        # whole 256-row blocks of the global A, generated once each
        out = np.empty((len(idx), size), np.int8)
        blocks = {}
        for j, r in enumerate(idx):
            b = r // BLOCK_ROWS
            if b not in blocks:
                blocks[b] = gen_rows(SEED_A, b * BLOCK_ROWS, min(size, (b + 1) * BLOCK_ROWS), size, 1).numpy()
            out[j] = blocks[b][r - b * BLOCK_ROWS]
        return out

    n = cpu_sample_count(a_rows, BT, threads, min(args.cpu_seconds, 4.0))
    A_s = a_rows(sample_rows(size, n))
    n = A_s.shape[0]
    times = []
    kind = "reference"
    for i in range(args.warmup + args.steps):
        _, t, kind = cpu_reference_rows(A_s, BT, threads)
        if i >= args.warmup:
            times.append(t)
    ops = 2.0 * n * size * size
    mean_t = sum(times) / len(times)
    tops = ops / mean_t / 1e12
    sample = (f"{n} of {size} rows of C per step (the first {n // 2} and last {n - n // 2}; "
              f"{n}x{size}x{size} int8 MACs), {threads} threads")
    line = {
        "metric": METRIC, "value": tops, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "impl": "reference",
        "config": workload_config(size, world),
        "cpu_baseline": {"value": tops, "unit": "TOPS", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": tops, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------- our arm ----

def timed(stream, fn, steps, warmup, barrier):
    """Run fn warmup times, then `steps` times between events on `stream`
    (barrier + synchronize on both sides).  Returns (total ms, per-step ms)."""
    import torch
    for _ in range(max(warmup, 3)):
        fn()
    stream.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    t0.record(stream)
    for i in range(steps):
        ev[i][0].record(stream)
        fn()
        ev[i][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return t0.elapsed_time(t1), [a.elapsed_time(b) for a, b in ev]


def pcie_copy_floor(A_h, B_h, C_h, rank, world, dev, stream, barrier, max_over_ranks, reps=3):
    """Milliseconds per step for the end-to-end step's host<->device bytes
    alone: this rank's pinned A rows and its 1/world share of B copied in on
    one stream while its pinned C rows are copied out on another, every rank
    at once (they share the host's memory and PCIe).  Max over ranks; the
    floor any host-buffer GEMM of this size reaches on this machine."""
    import torch
    rows, size = A_h.shape
    share = size // world
    B_mine = B_h[rank * share:(rank + 1) * share]
    A_d = torch.empty_like(A_h, device=dev)
    B_d = torch.empty_like(B_mine, device=dev)
    C_d = torch.empty_like(C_h, device=dev)
    s_in = torch.cuda.Stream(device=dev)

    def step():
        s_in.wait_stream(stream)
        with torch.cuda.stream(s_in):
            A_d.copy_(A_h, non_blocking=True)
            B_d.copy_(B_mine, non_blocking=True)
        with torch.cuda.stream(stream):
            C_h.copy_(C_d, non_blocking=True)
        stream.wait_stream(s_in)

    step()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(reps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / reps
    del A_d, B_d, C_d
    torch.cuda.empty_cache()
    return ms


def gathered_legs(args, A, BT, r0, rows, size, world, dev, stream, barrier, max_over_ranks):
    """The optional all-gather of C (more than one GPU): the GEMM epilogue
    storing every tile into all ranks' C over NVLink (p2p), and block-cyclic
    row blocks all-gathered by NCCL while the next block multiplies (nccl).
    Each is timed like the headline step and its full gathered C checked by
    Freivalds' check against the full A."""
    import torch
    import torch.distributed as dist

    from tensorcoreptx_b200.dist import PeerGather, cyclic_row_blocks, gathered_gemm_int8
    from tensorcoreptx_b200.verify import freivalds_int8

    out = {}
    A_full = torch.empty((size, size), dtype=torch.int8, device=dev)
    dist.all_gather_into_tensor(A_full, A)
    sent = rows * size * 4 * (world - 1)
    ops = 2.0 * size ** 3
    peer = PeerGather(size, size, dev)
    with torch.cuda.stream(stream):
        total, _ = timed(stream, lambda: peer.gemm_int8(A, BT, r0), args.steps, args.warmup, barrier)
    ms = max_over_ranks(total) / args.steps
    ok = freivalds_int8(A_full, BT, peer.C)
    bad = max_over_ranks(0.0 if ok else 1.0)
    out["gather_p2p"] = {"ms_per_step": ms, "tops": ops / ms / 1e9, "nvlink_bytes_sent_per_rank": sent,
                         "nvlink_bound_ms": sent / 770e9 * 1e3, "freivalds_pass": bad == 0.0}
    peer.close()
    del peer
    torch.cuda.empty_cache()
    chunks = 4
    A_cyc = torch.cat([A_full[b0:b1] for b0, b1 in cyclic_row_blocks(size, world, dist.get_rank(), chunks)])
    C_full = torch.empty((size, size), dtype=torch.int32, device=dev)
    with torch.cuda.stream(stream):
        total, _ = timed(stream, lambda: gathered_gemm_int8(A_cyc, BT, chunks, out=C_full), args.steps,
                         args.warmup, barrier)
    ms = max_over_ranks(total) / args.steps
    ok = freivalds_int8(A_full, BT, C_full)
    bad = max_over_ranks(0.0 if ok else 1.0)
    out["gather_nccl"] = {"ms_per_step": ms, "tops": ops / ms / 1e9, "nvlink_bytes_sent_per_rank": sent,
                          "nvlink_bound_ms": sent / 770e9 * 1e3, "freivalds_pass": bad == 0.0}
    del A_full, A_cyc, C_full
    torch.cuda.empty_cache()
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    import tensorcoreptx_b200 as T

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from tensorcoreptx_b200.dist import max_over_ranks as _max_over_ranks
    from tensorcoreptx_b200.dist import shard_rows
    from tensorcoreptx_b200.verify import freivalds_int8, rows_int8

    size = args.size
    r0, r1 = shard_rows(size, world, rank, align=256)
    rows = r1 - r0
    gather = args.gather if world > 1 else "none"
    if (gather != "none" or (world > 1 and not args.no_extras)) and size % (world * 4 * 256):
        raise SystemExit("the gathered steps need the rows to split into 4 equal 256-row blocks per rank")
    ops_total = 2.0 * size * size * size
    ops_rank = 2.0 * rows * size * size

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        return _max_over_ranks(x, device=dev)

    # inputs: this rank's rows of A and all of BT (N x K), generated on the
    # host, kept pinned for the end-to-end leg and copied to the device once.
    # With more than one GPU, A, B and C live in host memory shared by the
    # ranks (each rank generates its equal share of A's and B's rows), so
    # the end-to-end step can hand rows to whichever GPUs have the fastest
    # path to host memory.
    threads = max(1, host_threads() // world)
    shared = None
    if world > 1:
        import shutil
        need = 6 * size * size  # A and B int8, C int32
        try:
            room = shutil.disk_usage("/dev/shm").free >= 1.1 * need
        except OSError:
            room = False
        if max_over_ranks(0.0 if room else 1.0) == 0.0:
            from tensorcoreptx_b200.dist import SharedHostTensor
            shared = {"A": SharedHostTensor((size, size), torch.int8, tag="A"),
                      "B": SharedHostTensor((size, size), torch.int8, tag="B"),
                      "C": SharedHostTensor((size, size), torch.int32, tag="C")}
            gen_rows(SEED_A, r0, r1, size, threads, out=shared["A"].tensor[r0:r1])
            gen_rows(SEED_B, r0, r1, size, threads, out=shared["B"].tensor[r0:r1])
            barrier()
            A_h = shared["A"].tensor[r0:r1]
            B_h = shared["B"].tensor
    if shared is None:
        A_h = gen_rows(SEED_A, r0, r1, size, threads).pin_memory()
        B_h = gen_rows(SEED_B, 0, size, size, threads).pin_memory()
    A = A_h.to(dev)
    BT = B_h.to(dev)
    C = torch.empty(rows, size, dtype=torch.int32, device=dev)
    C_full = torch.empty(size, size, dtype=torch.int32, device=dev) if gather == "nccl" else None
    peer = None
    if gather == "p2p":
        from tensorcoreptx_b200.dist import PeerGather
        peer = PeerGather(size, size, dev)

    from tensorcoreptx_b200 import _native as nat
    lib = nat.lib()
    stream = torch.cuda.Stream(device=dev)
    nccl_chunks = 4
    A_step = A
    if gather == "nccl":
        from tensorcoreptx_b200.dist import cyclic_row_blocks, gathered_gemm_int8
        A_all = torch.empty((size, size), dtype=torch.int8, device=dev)
        dist.all_gather_into_tensor(A_all, A)
        A_step = torch.cat([A_all[b0:b1] for b0, b1 in cyclic_row_blocks(size, world, rank, nccl_chunks)])
        del A_all

    def step():
        if gather == "nccl":
            with torch.cuda.stream(stream):
                gathered_gemm_int8(A_step, BT, nccl_chunks, out=C_full)
            return
        if peer is not None:
            with torch.cuda.stream(stream):
                peer.gemm_int8(A, BT, r0)  # GEMM + epilogue stores to every rank + 1-word barrier
            return
        st = lib.tcg_gemm_s8(A.data_ptr(), BT.data_ptr(), C.data_ptr(), rows, size, size, 1,
                             nat.TCG_B_NK, stream.cuda_stream)
        nat.check("tcg_gemm_s8", st)

    clocks = ClockSampler(list(range(world)) if rank == 0 else [local])
    if rank == 0:
        clocks.start()
        time.sleep(0.5)

    # ---- kernel-resident timed region
    clocks.mark("warmup")
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
    stream.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    clocks.mark("kernel")
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_begin.record(stream)
    for i in range(args.steps):
        # with a gather the bracket holds the whole step (GEMM and transfer)
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks.mark(None)
    total_ms = max_over_ranks(t_begin.elapsed_time(t_end))
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    kern_ms = max_over_ranks(sum(launch_ms) / len(launch_ms))
    tile_n = T.last_tile_n()
    tile_m = T.last_tile_m()
    werr = T.check_device_error(stream)
    assert werr == 0

    # ---- parity of what was timed (outside the timed region)
    if gather == "nccl":
        C_mine = C_full
        A_chk = torch.empty((size, size), dtype=torch.int8, device=dev)
        dist.all_gather_into_tensor(A_chk, A)
    elif gather == "p2p":
        C_mine, A_chk = peer.C, None
        A_chk = torch.empty((size, size), dtype=torch.int8, device=dev)
        dist.all_gather_into_tensor(A_chk, A)
    else:
        C_mine, A_chk = C, A
    fv_ok = freivalds_int8(A_chk, BT, C_mine, trials=2, seed=rank)
    chk_rows = sorted({0, 1, C_mine.shape[0] - 2, C_mine.shape[0] - 1})
    rows_ok = bool(torch.equal(rows_int8(A_chk, BT, chk_rows), C_mine[chk_rows]))
    del A_chk
    if gather != "none":  # the e2e leg and the reference rows compare against the plain slice
        with torch.cuda.stream(stream):
            nat.check("tcg_gemm_s8", lib.tcg_gemm_s8(A.data_ptr(), BT.data_ptr(), C.data_ptr(), rows, size,
                                                     size, 1, nat.TCG_B_NK, stream.cuda_stream))
        stream.synchronize()
    if peer is not None:
        peer.close()
        del peer
    C_full = None
    torch.cuda.empty_cache()

    # ---- clock-normalised kernel rate: time x median SM clock, TOPS per GHz
    ksum = clocks.summary("kernel")
    mhz = ksum.get("sm_mhz")
    achieved = ops_rank / (kern_ms * 1e-3) / 1e12
    clock_norm = None
    if mhz:
        clock_norm = {"sm_mhz_median": mhz, "kernel_ms_x_ghz": kern_ms * mhz / 1e3,
                      "tops_per_ghz_per_gpu": achieved / (mhz / 1e3),
                      "note": "per-GPU kernel TOPS divided by the median SM clock of the timed window; "
                              "comparable across N with the power cap removed"}

    # ---- the gathered steps (N > 1), timed and checked as extras
    gathered = None
    if world > 1 and not args.no_extras:
        gathered = gathered_legs(args, A, BT, r0, rows, size, world, dev, stream, barrier, max_over_ranks)

    # ---- end-to-end through the public API: pinned host in, pinned host out
    group = dist.group.WORLD if world > 1 else None
    del A, BT
    torch.cuda.empty_cache()
    split = [shard_rows(size, world, k, align=256) for k in range(world)]
    if shared is not None:
        C_all = shared["C"].tensor
    else:
        C_h = torch.empty(rows, size, dtype=torch.int32).pin_memory()

    def e2e_step(a0, a1):
        # public host-buffer entry: pinned rows of A and B in (1/G of B per
        # rank plus an NVLink all-gather when G > 1), pinned rows of C out,
        # row x column blocks of C pipelined against the copies
        if shared is not None:
            T.gemm_int8_host(shared["A"].tensor[a0:a1], B_h, out=C_all[a0:a1], chunks=8, group=group)
        else:
            T.gemm_int8_host(A_h, B_h, out=C_h, chunks=8, group=group)

    calib = []
    if shared is not None:
        # The ranks' paths to host memory differ (on some nodes half the GPUs
        # reach it at a fraction of the others' rate) and share the host's
        # bandwidth, which more concurrent GPUs can lower.  So the rows of the
        # end-to-end step go to a set of ranks -- all of them, or the fastest
        # half or quarter by the rate each reached with all of them -- in
        # proportion to the rate each reaches on the step itself (a few damped
        # rounds per set), and the set whose step ended soonest is kept.
        # Ranks without rows still take part in gathering B.
        from tensorcoreptx_b200.dist import choose_host_rows

        def timed_rows(b0, b1):
            c0 = torch.cuda.Event(enable_timing=True)
            c1 = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                c0.record(stream)
                e2e_step(b0, b1)
                c1.record(stream)
            torch.cuda.synchronize()
            return c0.elapsed_time(c1)

        split, calib = choose_host_rows(size, timed_rows, device=dev, align=256, rounds=3)
    a0, a1 = split[rank]
    # before the end-to-end steps: it writes C rows, which they then overwrite
    if shared is not None:
        copy_floor_ms = pcie_copy_floor(shared["A"].tensor[a0:a1], B_h, C_all[a0:a1], rank, world, dev, stream,
                                        barrier, max_over_ranks)
    else:
        copy_floor_ms = pcie_copy_floor(A_h, B_h, C_h, rank, world, dev, stream, barrier, max_over_ranks)

    # Consecutive steps are issued on two streams in turn, as a caller with
    # independent requests would: each call is ordered after the previous
    # call on its own stream only, so one step's input copies can run while
    # the step before it is still copying C out (the library keeps every
    # call's outbound copies in order on its own copy stream).
    streams = [stream, torch.cuda.Stream(device=dev)]
    for i in range(max(args.warmup, 3)):
        with torch.cuda.stream(streams[i % 2]):
            e2e_step(a0, a1)
    torch.cuda.synchronize()
    e2e_steps = max(3, min(args.steps, 10))
    barrier()
    torch.cuda.synchronize()
    clocks.mark("e2e")
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    streams[1].wait_stream(stream)
    for i in range(e2e_steps):
        with torch.cuda.stream(streams[i % 2]):
            e2e_step(a0, a1)
    stream.wait_stream(streams[1])
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks.mark(None)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
    # bytes of the whole job per step: A and B once, C once
    h2d = 2 * size * size
    d2h = 4 * size * size
    if shared is not None and a1 == a0:
        e2e_ok = True  # no rows here: the other ranks' checks cover every row of C
        C_h = C_all[r0:r1]
    elif shared is not None:
        # this rank's end-to-end rows: Freivalds' check against its rows of A
        # and B, plus its first and last row recomputed in float64
        A_chk = shared["A"].tensor[a0:a1].to(dev)
        B_chk = B_h.to(dev)
        C_chk = C_all[a0:a1].to(dev)
        e2e_ok = freivalds_int8(A_chk, B_chk, C_chk, trials=2, seed=100 + rank)
        last = sorted({0, a1 - a0 - 1})
        e2e_ok = e2e_ok and bool(torch.equal(rows_int8(A_chk, B_chk, last), C_chk[last]))
        del A_chk, B_chk, C_chk
        C_h = C_all[r0:r1]
    else:
        e2e_ok = bool(torch.equal(C_h.to(dev), C))
    del C
    torch.cuda.empty_cache()

    if rank == 0:
        clocks.stop()
    bad = max_over_ranks(0.0 if (fv_ok and rows_ok and e2e_ok) else 1.0)
    parity = {"freivalds_trials": 2, "freivalds_pass": fv_ok, "rows_fp64_device": len(chk_rows),
              "rows_fp64_device_pass": rows_ok, "e2e_pass": e2e_ok,
              "all_ranks_pass": bad == 0.0,
              "what": "every rank: its whole C slice by Freivalds' check (C x == A (B^T x), exact in "
                      "float64), rows 0, 1, last-1, last recomputed in float64 on the GPU, and the "
                      "end-to-end C: equal to the resident C at one GPU; with more GPUs each rank's "
                      "end-to-end rows by Freivalds' check and their first and last row in float64"}
    parity["pass"] = parity["all_ranks_pass"]

    result = None
    if rank == 0:
        peaks, peak_src = load_peaks()
        # int8 dense tensor peak = 2x the dense bf16 peak on B200 (4.5 POPS vs
        # 2.25 PFLOP/s nominal).  The kernel is timed alone, back to back, so
        # the burst bf16 figure is the denominator.
        peak_tops = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
        traffic = profile_traffic(size, rows)
        ms_per_step = total_ms / args.steps
        result = {
            "metric": METRIC,
            "value": ops_total / (ms_per_step * 1e-3) / 1e12,
            "unit": "TOPS",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "int8",
            "data": "synthetic",
            "config": workload_config(size, world, gather),
            "tile": {"m": tile_m, "n": tile_n},
            "roofline": {
                "bound": "tensor",
                "achieved": achieved,
                "peak": peak_tops,
                "unit": "TOPS",
                "frac": achieved / peak_tops,
                "traffic": traffic,
                "peak_source": f"2 x bf16_tflops (burst) of MEASURED_PEAKS.json ({peak_src})",
                "frac_of_sustained": achieved / (2.0 * float(peaks.get("bf16_tflops_sustained", 1400.0))),
            },
            "e2e": {"value": ops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "bytes": "whole job per step: A and B in once, C out once",
                    "host_buffers": "private" if shared is None else "shared by the ranks (/dev/shm, pinned)",
                    "rows_per_rank": [b1 - b0 for b0, b1 in split],
                    "balance_rounds": calib,
                    "ms_per_step": e2e_ms,
                    "streams": "consecutive steps on two streams in turn (a step's inputs may copy in "
                               "while the previous step's C copies out)",
                    "copy_floor_ms": copy_floor_ms,
                    "frac_of_copy_floor": copy_floor_ms / e2e_ms,
                    "copy_floor": "the same host<->device bytes per rank with no GEMM: the rank's pinned "
                                  "rows of A and its share of B in, its pinned rows of C out, the two "
                                  "directions on two streams at once (max over ranks)"},
            "gpu_launches": args.steps * (nccl_chunks if gather == "nccl" else 1),
            "clocks": ksum,
            "clock_norm": clock_norm,
            "clocks_e2e": clocks.summary("e2e"),
            "parity": parity,
        }
        if gathered is not None:
            result["extras"] = gathered

    if world > 1:
        dist.barrier()
        if shared is not None:
            for sh in shared.values():
                sh.close()
        dist.destroy_process_group()
    return result, (A_h, B_h, C_h)


def profile_traffic(size, rows):
    """DRAM bytes per launch from the committed ncu capture of this kernel
    (profiles/gemm_s8_traffic.json): exact for the captured shape; for other
    per-rank shapes read bytes are scaled by MACs and write bytes by outputs.
    None when absent."""
    path = os.path.join(ROOT, "profiles", "gemm_s8_traffic.json")
    try:
        with open(path) as f:
            p = json.load(f)
        if (rows, size, size) == (p["M"], p["N"], p["K"]):
            return float(p["dram_read_bytes_per_launch"]) + float(p["dram_write_bytes_per_launch"])
        rd = float(p["dram_read_bytes_per_launch"]) / float(p["macs_per_launch"])
        wr = float(p["dram_write_bytes_per_launch"]) / float(p["outputs_per_launch"])
        return rd * rows * size * size + wr * rows * size
    except (OSError, ValueError, KeyError):
        return None


# ----------------------------------------------------------- extras (N=1) ----

def time_fn(fn, iters, pause=0.5):
    """Mean ms per call on the current stream after 3 warm-ups.  Every
    configuration starts from an idle GPU: without the pause, one timed right
    after a long power-capped loop inherits its clocks."""
    import torch
    torch.cuda.synchronize()
    time.sleep(pause)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def extras():
    """Kernel-only throughput of the other benchmark configurations on this
    GPU, for context (one-GPU runs only)."""
    import torch

    import tensorcoreptx_b200 as T

    dev = torch.device("cuda", 0)
    out = {}
    g = torch.Generator(device=dev).manual_seed(0)
    n = 4096
    A = torch.randint(-128, 128, (n, n), generator=g, device=dev, dtype=torch.int8)
    BT = torch.randint(-128, 128, (n, n), generator=g, device=dev, dtype=torch.int8)
    ms = time_fn(lambda: T.gemm_int8(A, BT), 50)
    out["int8_4096"] = {"tops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    try:
        ms_lib = time_fn(lambda: torch._int_mm(A, BT.t()), 50)
        out["int8_4096_torch_int_mm"] = {"tops": 2 * n ** 3 / ms_lib / 1e9, "ms": ms_lib}
    except Exception as e:  # pragma: no cover
        out["int8_4096_torch_int_mm"] = {"error": str(e)[:80]}
    # the same with B row-major (K x N), the layout the configuration names
    B_kn = BT.t().contiguous()
    ms = time_fn(lambda: T.gemm_int8_kn(A, B_kn), 50)
    out["int8_4096_b_row_major"] = {"tops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    del B_kn
    Ap = torch.randint(-128, 128, (n, n // 2), generator=g, device=dev, dtype=torch.int8)
    Bp = torch.randint(-128, 128, (n, n // 2), generator=g, device=dev, dtype=torch.int8)
    ms = time_fn(lambda: T.gemm_int4(Ap, Bp), 50)
    out["int4_4096"] = {"tops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    del A, BT, Ap, Bp
    # smallest sizes first and both accumulation modes per size: a size timed
    # right after a power-capped 16384^3 loop would run at reduced clocks
    for n in (512, 1024, 2048, 4096, 8192, 16384):
        A = (torch.rand(n, n, generator=g, device=dev) * 2 - 1).half()
        B = (torch.rand(n, n, generator=g, device=dev) * 2 - 1).half()
        iters = 50 if n <= 4096 else 10
        for acc in ("fp32", "fp16"):
            ms = time_fn(lambda: T.gemm_fp16(A, B, acc=acc), iters)
            out[f"fp16_{acc}acc_{n}"] = {"tflops": 2 * n ** 3 / ms / 1e9, "ms": ms}
        if n in (512, 4096, 16384):
            ms_lib = time_fn(lambda: torch.matmul(A, B), iters)
            out[f"fp16_{n}_torch_matmul"] = {"tflops": 2 * n ** 3 / ms_lib / 1e9, "ms": ms_lib}
        del A, B
    torch.cuda.empty_cache()
    # the rows beyond the benchmark configurations: FP8, the fused dequant
    # epilogue, on-device quantisation and the batched entry
    n = 4096
    for n8 in (4096, 8192):
        A8 = (torch.rand(n8, n8, generator=g, device=dev) * 2 - 1).to(torch.float8_e4m3fn)
        B8 = (torch.rand(n8, n8, generator=g, device=dev) * 2 - 1).to(torch.float8_e4m3fn)
        ms = time_fn(lambda: T.gemm_fp8(A8, B8), 20)
        out[f"fp8_e4m3_{n8}"] = {"tflops": 2 * n8 ** 3 / ms / 1e9, "ms": ms}
        try:
            one = torch.ones(1, device=dev)
            ms_lib = time_fn(lambda: torch._scaled_mm(A8, B8.t(), scale_a=one, scale_b=one,
                                                      out_dtype=torch.float32), 20)
            out[f"fp8_e4m3_{n8}_torch_scaled_mm"] = {"tflops": 2 * n8 ** 3 / ms_lib / 1e9, "ms": ms_lib}
        except Exception as e:  # pragma: no cover
            out[f"fp8_e4m3_{n8}_torch_scaled_mm"] = {"error": str(e)[:80]}
        del A8, B8
    Af = torch.randn(n, n, generator=g, device=dev)
    Bf = torch.randn(n, n, generator=g, device=dev)
    qa, sa = T.quantize_absmax_int8(Af)
    qb, sb = T.quantize_absmax_int8(Bf)
    ms = time_fn(lambda: T.gemm_int8_dequant(qa, qb, sa, sb), 50)
    out["int8_4096_dequant_fused"] = {"tops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    ms = time_fn(lambda: T.gemm_int8(qa, qb).float() * (sa * sb), 50)
    out["int8_4096_then_torch_dequant"] = {"tops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    del Af, Bf, qa, qb
    # quantisation: HBM-bound; algorithmic bytes = fp32 read once + codes
    # written (int8: 5 bytes per value, int4: 4.5); 256 MB of fp32, beyond L2
    hbm = float(load_peaks()[0].get("hbm_gbs", 6650.0))
    Xq = torch.randn(8192, 8192, generator=g, device=dev)
    for name, fn, per in (("quantize_int8_8192x8192", lambda: T.quantize_absmax_int8(Xq), 5.0),
                          ("quantize_int4_8192x8192", lambda: T.quantize_absmax_int4(Xq), 4.5)):
        ms = time_fn(fn, 20)
        gbs = per * Xq.numel() / ms / 1e6
        out[name] = {"gbs": gbs, "ms": ms, "frac_hbm": gbs / hbm}
    del Xq
    # batched: the reference profiles num_batches = 4
    Ab = (torch.rand(4, 2048, 2048, generator=g, device=dev) * 2 - 1).half()
    Bb = (torch.rand(4, 2048, 2048, generator=g, device=dev) * 2 - 1).half()
    ms = time_fn(lambda: T.gemm_fp16(Ab, Bb), 30)
    out["fp16_batched_4x2048"] = {"tflops": 4 * 2 * 2048 ** 3 / ms / 1e9, "ms": ms}
    ms_lib = time_fn(lambda: torch.bmm(Ab, Bb), 30)
    out["fp16_batched_4x2048_torch_bmm"] = {"tflops": 4 * 2 * 2048 ** 3 / ms_lib / 1e9, "ms": ms_lib}
    del Ab, Bb
    torch.cuda.empty_cache()
    # the smallest configuration (fp16 512^3) is launch-bound from Python;
    # its device time, from 20 launches replayed in a CUDA graph
    n = 512
    A = (torch.rand(n, n, generator=g, device=dev) * 2 - 1).half()
    B = (torch.rand(n, n, generator=g, device=dev) * 2 - 1).half()
    C = torch.empty(n, n, dtype=torch.float32, device=dev)
    from tensorcoreptx_b200 import _native as nat
    L = nat.lib()
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        for _ in range(3):
            nat.check("fp16", L.tcg_gemm_f16(A.data_ptr(), B.data_ptr(), C.data_ptr(), n, n, n, 1,
                                             nat.TCG_ACC_F32, nat.TCG_B_KN, s.cuda_stream))
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for _ in range(20):
            nat.check("fp16", L.tcg_gemm_f16(A.data_ptr(), B.data_ptr(), C.data_ptr(), n, n, n, 1,
                                             nat.TCG_ACC_F32, nat.TCG_B_KN, s.cuda_stream))
    ms = time_fn(graph.replay, 20) / 20
    out["fp16_fp32acc_512_graph"] = {"tflops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    del graph
    return out


# --------------------------------------------- reported baselines (N=1) ----
#
# Everything below runs after the timed regions and only reports: the
# reference's own code (its CPU GEMM and its GPU kernels, compiled unchanged
# into oracle/_ref/) and a blocked CPU GEMM, each on this box.

def cpu_baseline_leg(args, A_h, B_h, C_h):
    """The reference's cpu_gemm_int8 on a row sample of this run's own inputs
    (all host threads), timed -- and its rows compared with the GPU's C rows
    of the same inputs (the row-level parity of the headline config)."""
    import numpy as np
    size = args.size
    threads = host_threads()
    A_np = A_h.numpy()
    B_np = B_h.numpy()

    def a_rows(idx):
        return np.ascontiguousarray(A_np[idx])

    n = cpu_sample_count(a_rows, B_np, threads, args.cpu_seconds)
    idx = sample_rows(A_np.shape[0], n)
    ref, t, kind = cpu_reference_rows(a_rows(idx), B_np, threads)
    n = len(idx)
    ok = bool(np.array_equal(ref, C_h.numpy()[idx]))
    line = {"value": 2.0 * n * size * size / t / 1e12, "unit": "TOPS", "cores": threads, "kind": kind,
            "sample": f"{n} of {size} rows of C (the first {n // 2} and last {n - n // 2} of this run's own "
                      f"inputs; {n}x{size}x{size} int8 MACs) in {t:.1f} s"}
    return line, {"rows_vs_reference_cpu": n, "rows_vs_reference_cpu_pass": ok,
                  "reference_cpu_kind": kind}


def blocked_cpu_leg():
    """The blocked multi-threaded CPU GEMM (oracle/cpu_blocked.c) on all host
    threads: fp16 512^3, int8 4096^3, int4 4096^3 (best of 3)."""
    import numpy as np
    from oracle import oracle as O
    threads = host_threads()
    rng = np.random.default_rng(0)
    out = {"cores": threads, "what": "cache-blocked AVX2 CPU GEMM, all host threads, best of 3"}

    def best(fn):
        fn()
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return min(ts)

    n = 512
    Ah = rng.uniform(-1, 1, (n, n)).astype(np.float16).view(np.uint16)
    Bh = rng.uniform(-1, 1, (n, n)).astype(np.float16).view(np.uint16)
    t = best(lambda: O.blocked_gemm_f16(Ah, Bh, threads=threads))
    out["fp16_512"] = {"tflops": 2 * n ** 3 / t / 1e12, "ms": t * 1e3}
    n = 4096
    A8 = rng.integers(-128, 128, (n, n), dtype=np.int8)
    B8 = rng.integers(-128, 128, (n, n), dtype=np.int8)
    t = best(lambda: O.blocked_gemm_s8(A8, B8, threads=threads))
    out["int8_4096"] = {"tops": 2 * n ** 3 / t / 1e12, "ms": t * 1e3}
    A4 = rng.integers(-128, 128, (n, n // 2), dtype=np.int8)
    B4 = rng.integers(-128, 128, (n, n // 2), dtype=np.int8)
    t = best(lambda: O.blocked_gemm_s4(A4, B4, n, threads=threads))
    out["int4_4096"] = {"tops": 2 * n ** 3 / t / 1e12, "ms": t * 1e3}
    return out


def naive_reference_cpu_leg():
    """The reference's own CPU GEMMs (src/data.cu cpu_gemm_fp16,
    src/data_int8.cu cpu_gemm_int8, src/data_int4.cu cpu_gemm_int4, compiled
    unchanged into oracle/_ref/) at 512^3 on one host thread, on the
    reference's own seeded inputs (its generate_* functions): the naive loop
    the reference checks its kernels with, for context beside the blocked
    GEMM.  Empty when the reference was not built here."""
    import numpy as np
    from oracle import oracle as O
    n = 512
    out = {"threads": 1, "what": "reference cpu_gemm_* (naive i-j-k), one call each"}
    for which, abytes, key, unit in (("fp16", 2 * n, "fp16_512", "tflops"), ("int8", n, "int8_512", "tops"),
                                      ("int4", n // 2, "int4_512", "tops")):
        L = O.ref_data_lib(which)
        if L is None:
            return {}
        A = np.zeros(n * abytes, np.uint8)
        B = np.zeros(n * abytes, np.uint8)
        Cm = np.zeros(n * n, np.float32 if which == "fp16" else np.int32)
        L.gen(A.ctypes.data, B.ctypes.data, n, n, n, 1)
        t0 = time.perf_counter()
        L.gemm(A.ctypes.data, B.ctypes.data, Cm.ctypes.data, n, n, n)
        t = time.perf_counter() - t0
        out[key] = {unit: 2 * n ** 3 / t / 1e12, "ms": t * 1e3}
    return out


def reference_kernels_leg():
    """The reference's GPU kernels recompiled unchanged for sm_100a
    (oracle/_ref/libref_<kernel>.so), timed on this B200 like ours: int8 and
    int4 at 4096^3, fp16 at 512^3 and 4096^3."""
    import torch
    from oracle import ref_kernels as RK
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    out = {}
    n = 4096
    A = torch.randint(-128, 128, (n, n), generator=g, device=dev, dtype=torch.int8)
    B = torch.randint(-128, 128, (n, n), generator=g, device=dev, dtype=torch.int8)
    for name in ("int8_wmma", "int8_ptx_mma_k32"):
        if RK.available(name):
            ms = time_fn(lambda: RK.run(name, A, B, n, n, n), 10)
            out[f"{name}_4096"] = {"tops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    Ap, Bp = A[:, :n // 2].contiguous(), B[:, :n // 2].contiguous()
    for name in ("int4_wmma", "int4_ptx_mma_k64_x4_x2nontrans_ca"):
        if RK.available(name):
            ms = time_fn(lambda: RK.run(name, Ap, Bp, n, n, n), 10)
            out[f"{name}_4096"] = {"tops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    del A, B, Ap, Bp
    for n in (512, 4096):
        Ah = (torch.rand(n, n, generator=g, device=dev) * 2 - 1).half()
        Bh = (torch.rand(n, n, generator=g, device=dev) * 2 - 1).half()
        for name in ("fp16_wmma", "fp16_ptx_fp16acc"):
            if RK.available(name):
                ms = time_fn(lambda: RK.run(name, Ah, Bh, n, n, n), 10 if n > 512 else 50)
                out[f"{name}_{n}"] = {"tflops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    torch.cuda.empty_cache()
    return out


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    # Libraries (NCCL's version banner, for one) may print to stdout; keep
    # stdout for the one JSON line by sending everything else to stderr.
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    result, host = run_ours(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank == 0 and result is not None:
        if world == 1 and not args.no_cpu_baseline:
            line, rows = cpu_baseline_leg(args, *host)
            result["cpu_baseline"] = line
            result["parity"].update(rows)
            result["parity"]["pass"] = result["parity"]["pass"] and rows["rows_vs_reference_cpu_pass"]
        del host
        if world == 1 and not args.no_extras:
            ex = extras()
            ex["reference_kernels_b200"] = reference_kernels_leg()
            if not args.no_cpu_baseline:
                ex["cpu_blocked"] = blocked_cpu_leg()
                ex["cpu_reference_naive"] = naive_reference_cpu_leg()
            result["extras"] = ex
        sys.stdout.flush()
        os.write(json_fd, (json.dumps(result) + "\n").encode())
    return 0


if __name__ == "__main__":
    sys.exit(main())
