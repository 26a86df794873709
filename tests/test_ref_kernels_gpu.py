"""The reference's own kernels, recompiled unchanged for sm_100a
(oracle/_ref/), on the same B200: their verify case against the oracle (the
same bar our kernels meet), and their speed against ours on the benchmark
shapes.  Timings go to $TCG_RESULTS_DIR/gpu_results.json when that is set."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

from oracle import ref_kernels as RK

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _record(key, value):
    d = os.environ.get("TCG_RESULTS_DIR")
    if not d:
        return
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, "gpu_results.json")
    data = json.load(open(path)) if os.path.exists(path) else {}
    data[key] = value
    json.dump(data, open(path, "w"), indent=1, sort_keys=True)


def _need(name):
    if not RK.available(name):
        pytest.skip(f"oracle/_ref/libref_{name}.so not built")


def _time_ms(fn, iters=20):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


@pytest.mark.parametrize("name", ["int8_wmma", "int8_ptx_mma_k32"])
def test_reference_int8_kernel_verify_512(name):
    _need(name)
    A, BT = O.generate_int8(512, 512, 512)
    C = RK.run(name, torch.from_numpy(A[0]).to(DEV), torch.from_numpy(BT[0]).to(DEV),
               512, 512, 512).cpu().numpy()
    acc = O.measure_accuracy_i32(O.gemm_s8(A[0], BT[0], threads=8), C)
    assert acc.pass_ and C[0, 0] == -149768


@pytest.mark.parametrize("name", ["int4_wmma", "int4_ptx_mma_k64_x4_x2nontrans_ca"])
def test_reference_int4_kernel_verify_512(name):
    _need(name)
    A, BT = O.generate_int4_packed(512, 512, 512)
    C = RK.run(name, torch.from_numpy(A[0]).to(DEV), torch.from_numpy(BT[0]).to(DEV),
               512, 512, 512).cpu().numpy()
    acc = O.measure_accuracy_i32(O.gemm_s4(A[0], BT[0], 512, threads=8), C)
    assert acc.pass_ and C[0, 0] == -563


def test_negative_control_reference_kernel_is_flagged():
    """The reference's known-wrong int4 kernel (x2_x2 ldmatrix mapping), run
    on the verify inputs: the checker must fail it exactly as the
    reference's own log did (max_abs 2363 at (304,455), ref 1182, out -1181)."""
    name = "int4_ptx_mma_k64_x2_x2nontrans_ca"
    _need(name)
    nc = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")))[
        "int4_negative_control"]
    A, BT = O.generate_int4_packed(512, 512, 512)
    C = RK.run(name, torch.from_numpy(A[0]).to(DEV), torch.from_numpy(BT[0]).to(DEV),
               512, 512, 512).cpu().numpy()
    acc = O.measure_accuracy_i32(O.gemm_s4(A[0], BT[0], 512, threads=8), C)
    assert not acc.pass_
    assert (acc.max_abs_err, acc.max_row, acc.max_col, acc.ref_at_max, acc.out_at_max) == \
        (nc["max_abs"], nc["row"], nc["col"], nc["ref"], nc["bad_out"])


@pytest.mark.parametrize("name", ["fp16_wmma", "fp16_ptx_fp16acc"])
def test_reference_fp16_kernel_within_same_tolerance(name):
    """The tolerance our fp16 path meets, applied to the reference's output."""
    _need(name)
    rng = np.random.default_rng(0)
    A = rng.uniform(-1, 1, (512, 512)).astype(np.float16).view(np.uint16)
    B = rng.uniform(-1, 1, (512, 512)).astype(np.float16).view(np.uint16)
    C = RK.run(name, torch.from_numpy(A).view(torch.float16).to(DEV),
               torch.from_numpy(B).view(torch.float16).to(DEV), 512, 512, 512).cpu().numpy()
    err = float(np.abs(C - O.gemm_f16_f64(A, B, threads=8)).max())
    assert err <= O.fp16_tolerance(A, B, 512)


def test_ours_vs_reference_kernels_speed():
    """Benchmark shapes on this B200: int8/int4 4096^3, fp16 512^3 and 4096^3."""
    import tensorcoreptx_b200 as T
    g = torch.Generator(device=DEV).manual_seed(0)
    res = {}
    n = 4096
    A = torch.randint(-128, 128, (n, n), generator=g, device=DEV, dtype=torch.int8)
    BT = torch.randint(-128, 128, (n, n), generator=g, device=DEV, dtype=torch.int8)
    res["int8_4096_ours_ms"] = _time_ms(lambda: T.gemm_int8(A, BT))
    for name in ("int8_wmma", "int8_ptx_mma_k32"):
        if RK.available(name):
            res[f"int8_4096_{name}_ms"] = _time_ms(lambda: RK.run(name, A, BT, n, n, n), 5)
    Ap = torch.randint(-128, 128, (n, n // 2), generator=g, device=DEV, dtype=torch.int8)
    Bp = torch.randint(-128, 128, (n, n // 2), generator=g, device=DEV, dtype=torch.int8)
    res["int4_4096_ours_ms"] = _time_ms(lambda: T.gemm_int4(Ap, Bp))
    for name in ("int4_wmma", "int4_ptx_mma_k64_x4_x2nontrans_ca"):
        if RK.available(name):
            res[f"int4_4096_{name}_ms"] = _time_ms(lambda: RK.run(name, Ap, Bp, n, n, n), 5)
    for n in (512, 4096):
        Ah = (torch.rand(n, n, generator=g, device=DEV) * 2 - 1).half()
        Bh = (torch.rand(n, n, generator=g, device=DEV) * 2 - 1).half()
        res[f"fp16_{n}_ours_ms"] = _time_ms(lambda: T.gemm_fp16(Ah, Bh))
        res[f"fp16acc16_{n}_ours_ms"] = _time_ms(lambda: T.gemm_fp16(Ah, Bh, acc="fp16"))
        for name in ("fp16_wmma", "fp16_ptx_fp16acc"):
            if RK.available(name):
                res[f"fp16_{n}_{name}_ms"] = _time_ms(lambda: RK.run(name, Ah, Bh, n, n, n), 5)
    _record("speed_vs_reference_kernels", res)
    print(json.dumps(res, indent=1))
    # ours must beat every recompiled reference kernel at 4096^3
    for prec in ("int8", "int4"):
        ours = res[f"{prec}_4096_ours_ms"]
        for k, v in res.items():
            if k.startswith(f"{prec}_4096_") and "_ours_" not in k:
                assert ours < v, (k, ours, v)
    for k, v in res.items():
        if k.startswith("fp16_4096_") and "_ours_" not in k:
            assert res["fp16_4096_ours_ms"] < v, (k, v)


@pytest.mark.parametrize("n", [512, 1024, 4096])
@pytest.mark.parametrize("acc,name", [("fp32", "fp16_wmma"), ("fp16", "fp16_ptx_fp16acc")])
def test_fp16_bit_identical_to_reference_kernels(n, acc, name):
    """Both accumulation modes reproduce the reference's own kernels
    (recompiled for sm_100a, same GPU, same inputs) bit for bit: each output
    is accumulated 16 k at a time in increasing k with the same rounding."""
    _need(name)
    import tensorcoreptx_b200 as T
    g = torch.Generator(device=DEV).manual_seed(n)
    A = (torch.rand(n, n, generator=g, device=DEV) * 2 - 1).half()
    B = (torch.rand(n, n, generator=g, device=DEV) * 2 - 1).half()
    ours = T.gemm_fp16(A, B, acc=acc)
    theirs = RK.run(name, A, B, n, n, n)
    assert torch.equal(ours.view(torch.int32), theirs.view(torch.int32))


@pytest.mark.parametrize("name", ["int8_wmma", "int8_ptx_mma_k32"])
def test_int8_identical_to_reference_kernels_4096(name):
    _need(name)
    import tensorcoreptx_b200 as T
    g = torch.Generator(device=DEV).manual_seed(1)
    A = torch.randint(-128, 128, (4096, 4096), generator=g, device=DEV, dtype=torch.int8)
    BT = torch.randint(-128, 128, (4096, 4096), generator=g, device=DEV, dtype=torch.int8)
    assert torch.equal(T.gemm_int8(A, BT), RK.run(name, A, BT, 4096, 4096, 4096))
