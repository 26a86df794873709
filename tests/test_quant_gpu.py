"""On-device absmax quantisation and the dequantising GEMM epilogue, checked
bit for bit against the oracle's restatement of the reference's host code,
and the reference's whole quantisation round trip (src/main_int8.cu:53-100,
src/main_int4.cu:52-90) run on the device against its logged numbers."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
KNOWN = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "known_answers.json")))


def T():
    import tensorcoreptx_b200 as t
    return t


@pytest.mark.parametrize("n", [1, 3, 4, 1000, 4097, 1 << 20, (1 << 24) + 3])
def test_quantize_int8_bit_exact(n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    q, s = T().quantize_absmax_int8(torch.from_numpy(x).to(DEV))
    qo, so = O.quantize_absmax_s8(x)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.float32(s.item()).view(np.uint32) == np.float32(so).view(np.uint32)


@pytest.mark.parametrize("rows,k", [(1, 2), (3, 10), (512, 512), (77, 130), (2048, 4098)])
def test_quantize_int4_bit_exact(rows, k):
    rng = np.random.default_rng(rows * k)
    x = (rng.standard_normal((rows, k)) * 2).astype(np.float32)
    q, s = T().quantize_absmax_int4(torch.from_numpy(x).to(DEV))
    qo, so = O.quantize_absmax_s4(x)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.float32(s.item()).view(np.uint32) == np.float32(so).view(np.uint32)


def test_all_zero_input_gives_zero_scale_and_codes():
    q, s = T().quantize_absmax_int8(torch.zeros(100, device=DEV))
    assert s.item() == 0.0 and int(q.abs().sum()) == 0


@pytest.mark.parametrize("prec", ["int8", "int4"])
def test_reference_quant_round_trip_on_device(prec):
    """fp32 N(0,1) inputs (srand(43)) -> device quantise -> tensor-core GEMM
    with fused dequantisation -> compare with the fp64 GEMM: the numbers the
    reference printed, digit for digit, because every step is bit-identical."""
    M = N = K = 512
    Af, Bf = O.generate_fp32_normal(M, N, K)
    ref = O.gemm_f32(Af[0], Bf[0])
    t = T()
    A = torch.from_numpy(Af[0]).to(DEV)
    B = torch.from_numpy(Bf[0]).to(DEV)
    if prec == "int8":
        qa, sa = t.quantize_absmax_int8(A)
        qb, sb = t.quantize_absmax_int8(B)
        out = t.gemm_int8_dequant(qa, qb, sa, sb).cpu().numpy()
        qao, sao = O.quantize_absmax_s8(Af[0])
        qbo, sbo = O.quantize_absmax_s8(Bf[0])
        host = O.dequantize(O.gemm_s8(qao, qbo, threads=8), sao, sbo)
        tol = 0.1
    else:
        qa, sa = t.quantize_absmax_int4(A)
        qb, sb = t.quantize_absmax_int4(B)
        out = t.gemm_int4_dequant(qa, qb, sa, sb).cpu().numpy()
        qao, sao = O.quantize_absmax_s4(Af[0])
        qbo, sbo = O.quantize_absmax_s4(Bf[0])
        host = O.dequantize(O.gemm_s4(qao, qbo, K, threads=8), sao, sbo)
        tol = 1.0
    assert np.array_equal(out.view(np.uint32), host.view(np.uint32))
    acc = O.measure_accuracy_quant(ref, out, tol)
    k = KNOWN[f"{prec}_quant"]
    assert f"{sa.item():.4e}" == k["scale_A"] and f"{sb.item():.4e}" == k["scale_BT"]
    assert f"{acc.max_abs_err:.4e}" == k["max_abs"] and f"{acc.rmse:.4e}" == k["rmse"]
    assert f"{acc.snr_db:.1f}" == k["snr_db"]


@pytest.mark.parametrize("M,N,K", [(300, 200, 256), (1024, 2048, 512), (3328, 2560, 128)])
def test_dequant_epilogue_every_shape(M, N, K):
    rng = np.random.default_rng(M)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    BT = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sa, sb = np.float32(0.0123), np.float32(3.5e-3)
    t = T()
    out = t.gemm_int8_dequant(torch.from_numpy(A).to(DEV), torch.from_numpy(BT).to(DEV),
                              torch.tensor([sa], device=DEV), torch.tensor([sb], device=DEV)).cpu().numpy()
    host = O.dequantize(O.gemm_s8(A, BT, threads=8), float(sa), float(sb))
    assert np.array_equal(out.view(np.uint32), host.view(np.uint32))
