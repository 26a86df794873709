#!/usr/bin/env python
"""Benchmark of the tensor-core GEMM path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the sharded int8 GEMM, M = N = K = 32768 in total, int8 uniform
[-128, 127] from a seed, int32 accumulation and output.  A is row-partitioned
across the ranks (M/G rows each), B is replicated, each rank computes its
M/G x N slice of C (no data-path collective; ``--gather`` adds the optional
all-gather of C).  The total problem is fixed, so scaling is "strong"; at one
GPU this is the full 32768^3 problem on one B200.

A "step" is one GEMM of each rank's slice.  ``value`` is whole-job TOPS with
inputs resident in HBM (inputs are 2 GiB, larger than L2, so no flush is
needed); ``e2e`` is the same metric through the public host-buffer API
(``gemm_int8_host``) with the step's A slice and B copied from pinned host
memory and its C slice copied back inside the timed region.  Device time is measured with CUDA events on
the launching stream, max over ranks.

``--impl reference`` times the reference's own CPU GEMM (src/data_int8.cu
cpu_gemm_int8, compiled unchanged into oracle/_ref/) on a bounded row sample
of the same workload with all host threads; only rank 0 runs it.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GEMM TFLOPS(fp16)/TOPS(int8,int4) per B200 + % dense tensor peak; 8-GPU agg"
SIZE = 32768


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--size", type=int, default=SIZE, help="M = N = K of the whole problem")
    ap.add_argument("--gather", choices=["none", "nccl", "p2p"], default="none",
                    help="all-gather C each step: NCCL after the GEMM, or peer stores from the "
                         "GEMM epilogue (p2p)")
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


# -------------------------------------------------------- reference (CPU) ----

_CPU_INPUTS = {}


def _cpu_inputs(size, rows):
    """Seeded int8 operands for the CPU sample: `rows` rows of A and all of
    BT (N x K), generated once per process."""
    import numpy as np
    if _CPU_INPUTS.get("size") != size:
        _CPU_INPUTS.clear()
        _CPU_INPUTS["size"] = size
        _CPU_INPUTS["BT"] = np.random.default_rng(1).integers(-128, 128, (size, size), dtype=np.int8)
    if _CPU_INPUTS.get("rows") != rows:
        _CPU_INPUTS["rows"] = rows
        _CPU_INPUTS["A"] = np.random.default_rng(0).integers(-128, 128, (rows, size), dtype=np.int8)
    return _CPU_INPUTS["A"], _CPU_INPUTS["BT"]


def cpu_reference_sample(size, rows, threads):
    """Run the reference's own cpu_gemm_int8 (oracle/_ref) -- or, when the
    reference was not available at build time, the oracle's restatement --
    on `rows` rows of C for the size^3 int8 problem.  Returns (seconds, kind)."""
    import numpy as np
    from oracle import oracle as O

    A, BT = _cpu_inputs(size, rows)
    Cs = np.zeros((rows, size), np.int32)
    t0 = time.perf_counter()
    if O.ref_data_lib("int8") is not None:
        O.ref_gemm_rows("int8", A, BT, rows, size, size, Cs, 0, rows, threads=threads)
        kind = "reference"
    else:
        Cs[:] = O.gemm_s8(A, BT, threads=threads)
        kind = "port"
    return time.perf_counter() - t0, kind


def cpu_sample_rows(size, threads, target_s):
    """Rows per sample so one sample takes about target_s seconds."""
    t, _ = cpu_reference_sample(size, threads, threads)  # one row per thread
    per_round = max(t, 1e-3)
    rounds = max(1, int(target_s / per_round))
    return threads * rounds


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    size = args.size
    threads = host_threads()
    rows = cpu_sample_rows(size, threads, min(args.cpu_seconds, 4.0))
    times = []
    kind = "reference"
    for i in range(args.warmup + args.steps):
        t, kind = cpu_reference_sample(size, rows, threads)
        if i >= args.warmup:
            times.append(t)
    ops = 2.0 * rows * size * size
    mean_t = sum(times) / len(times)
    tops = ops / mean_t / 1e12
    sample = f"{rows} of {size} rows of C per step ({rows}x{size}x{size} int8 MACs), {threads} threads"
    line = {
        "metric": METRIC, "value": tops, "unit": "TOPS", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": f"int8 GEMM M=N=K={size}, A row-sharded, B replicated, int32 C",
                   "parallelism": f"rows{args.gpus}"},
        "cpu_baseline": {"value": tops, "unit": "TOPS", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": tops, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------- our arm ----

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

    size = args.size
    r0, r1 = shard_rows(size, world, rank, align=256)
    rows = r1 - r0
    gather = args.gather if world > 1 else "none"
    if gather != "none" and size % world != 0:
        raise SystemExit("--gather needs the rows to divide evenly across ranks")
    ops_total = 2.0 * size * size * size
    ops_rank = 2.0 * rows * size * size

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        return _max_over_ranks(x, device=dev)

    # inputs: A slice of this rank, full B (BT layout, N x K), seeded on the GPU
    g = torch.Generator(device=dev).manual_seed(1234)
    A_full_seed_offset = rank  # each rank draws its own rows of the global A
    g.manual_seed(1234 + A_full_seed_offset)
    A = torch.randint(-128, 128, (rows, size), generator=g, device=dev, dtype=torch.int8)
    g.manual_seed(999)  # identical B on every rank (replicated)
    BT = torch.randint(-128, 128, (size, size), generator=g, device=dev, dtype=torch.int8)
    C = torch.empty(rows, size, dtype=torch.int32, device=dev)
    C_full = torch.empty(size, size, dtype=torch.int32, device=dev) if gather == "nccl" else None
    peer = None
    if gather == "p2p":
        from tensorcoreptx_b200.dist import PeerGather
        peer = PeerGather(size, size, dev)

    from tensorcoreptx_b200 import _native as nat
    lib = nat.lib()
    stream = torch.cuda.Stream(device=dev)

    def gemm_launch():
        if peer is not None:
            with torch.cuda.stream(stream):
                peer.gemm_int8(A, BT, r0)  # GEMM + epilogue stores to every rank + 1-word barrier
            return
        st = lib.tcg_gemm_s8(A.data_ptr(), BT.data_ptr(), C.data_ptr(), rows, size, size, 1,
                             nat.TCG_B_NK, stream.cuda_stream)
        nat.check("tcg_gemm_s8", st)

    # --gather nccl: block-cyclic row blocks, each multiplied into its place
    # in the full C and all-gathered in place while the next one multiplies
    nccl_chunks = 4
    if gather == "nccl" and rows % nccl_chunks:
        raise SystemExit("--gather nccl needs each rank's rows to split into 4 blocks")

    def step():
        if gather == "nccl":
            from tensorcoreptx_b200.dist import gathered_gemm_int8
            with torch.cuda.stream(stream):
                gathered_gemm_int8(A, BT, nccl_chunks, out=C_full)
            return
        gemm_launch()

    clocks = ClockSampler(list(range(world)) if rank == 0 else [local])
    if rank == 0:
        clocks.start()
        time.sleep(0.5)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
    stream.synchronize()

    # ---- kernel-resident timed region
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

    if peer is not None:
        peer.close()
        del peer
    # ---- end-to-end through the public API: pinned host in, pinned host out
    A_h = A.cpu().pin_memory()
    B_h = BT.cpu().pin_memory()
    C_h = torch.empty(rows, size, dtype=torch.int32).pin_memory()
    del A, BT, C
    torch.cuda.empty_cache()

    def e2e_step():
        # public host-buffer entry: pinned A slice and B in, pinned C slice out,
        # row chunks of C pipelined against the copies
        T.gemm_int8_host(A_h, B_h, out=C_h, chunks=8)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            e2e_step()
    stream.synchronize()
    e2e_steps = max(3, min(args.steps, 10))
    barrier()
    torch.cuda.synchronize()
    clocks.mark("e2e")
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks.mark(None)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
    h2d = rows * size + size * size
    d2h = rows * size * 4
    del A_h, B_h, C_h
    torch.cuda.empty_cache()

    if rank == 0:
        clocks.stop()

    result = None
    if rank == 0:
        peaks, peak_src = load_peaks()
        # int8 dense tensor peak = 2x the dense bf16 peak on B200 (4.5 POPS vs
        # 2.25 PFLOP/s nominal).  The kernel is timed alone, back to back, so
        # the burst bf16 figure is the denominator.
        peak_tops = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
        achieved = ops_rank / (kern_ms * 1e-3) / 1e12
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
            "config": {
                "workload": f"int8 GEMM M=N=K={size}, A row-sharded over {world} GPU(s), "
                            f"B replicated, int32 C" + {"none": "", "nccl": ", C all-gathered (NCCL, block-cyclic rows, "
                                                                 "4 blocks each gathered while the next "
                                                                 "multiplies)",
                                                         "p2p": ", C all-gathered by the GEMM epilogue "
                                                                "over NVLink peer stores"}[gather],
                "per_rank": f"{rows}x{size}x{size}",
                "values": "int8 uniform [-128,127], seeded",
                "l2": "inputs (2 GiB) larger than L2; no flush",
                "tile_m": tile_m,
                "tile_n": tile_n,
                "parallelism": f"rows{world}",
            },
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
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps * (nccl_chunks if gather == "nccl" else 1),
            "clocks": clocks.summary("kernel"),
            "clocks_e2e": clocks.summary("e2e"),
        }

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


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

def extras():
    """Kernel-only throughput of the other benchmark configurations on this
    GPU, for context (one-GPU runs only)."""
    import torch

    import tensorcoreptx_b200 as T

    dev = torch.device("cuda", 0)
    out = {}

    def time_fn(fn, iters):
        # every configuration starts from an idle GPU: without the pause, one
        # timed right after a long power-capped loop inherits its clocks
        torch.cuda.synchronize()
        time.sleep(0.5)
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
    ws = torch.empty(T.int4_workspace_size(n, n, n), dtype=torch.uint8, device=dev)
    ms = time_fn(lambda: T.gemm_int4(Ap, Bp, workspace=ws), 50)
    out["int4_4096"] = {"tops": 2 * n ** 3 / ms / 1e9, "ms": ms}
    del A, BT, Ap, Bp, ws
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


def cpu_baseline_line(args):
    size = args.size
    threads = host_threads()
    rows = cpu_sample_rows(size, threads, args.cpu_seconds)
    t, kind = cpu_reference_sample(size, rows, threads)
    return {"value": 2.0 * rows * size * size / t / 1e12, "unit": "TOPS", "cores": threads,
            "kind": kind,
            "sample": f"{rows} of {size} rows of C ({rows}x{size}x{size} int8 MACs) in {t:.1f} s"}


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    # Libraries (NCCL's version banner, for one) may print to stdout; keep
    # stdout for the one JSON line by sending everything else to stderr.
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    result = run_ours(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank == 0 and result is not None:
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline_line(args)
        if world == 1 and not args.no_extras:
            result["extras"] = extras()
        sys.stdout.flush()
        os.write(json_fd, (json.dumps(result) + "\n").encode())
    return 0


if __name__ == "__main__":
    sys.exit(main())
