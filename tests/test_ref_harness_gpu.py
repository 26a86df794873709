"""The reference's own executables -- src/main*.cu, src/solver*.cu and
src/data*.cu compiled unchanged (oracle/Makefile, target `harness`) and linked
against libtcgemm_compat_{f16,s8,s4}.so in place of a kernels/*.cu file --
run on the GPU: their own verify and quantisation lines must report what the
reference's logs report for its own kernels."""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref")


def _run(name, env):
    exe = os.path.join(BIN, name)
    if not os.path.exists(exe):
        pytest.skip(f"{name} not built (make -C oracle harness)")
    out = subprocess.run([exe], env={**os.environ, **env}, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return out.stdout


def test_reference_int8_harness_on_tcgemm():
    out = _run("ref_main_int8_on_tcgemm", {"SKIP_PROFILE": "1"})
    assert re.search(r"\[verify\]\s+M=512 N=512 K=512\s+PASS\s+max_abs=0 .* ref=-149768 out=-149768", out), out
    assert "scale_A=4.2262e-02 scale_BT=3.5921e-02" in out and "snr=35.9 dB" in out, out


def test_reference_int4_harness_on_tcgemm():
    out = _run("ref_main_int4_on_tcgemm", {"SKIP_PROFILE": "1"})
    assert re.search(r"\[verify\]\s+M=512 N=512 K=512\s+PASS\s+max_abs=0 .* ref=-563 out=-563", out), out
    assert "scale_A=7.6675e-01 scale_BT=6.5171e-01" in out and "snr=10.7 dB" in out, out


@pytest.mark.parametrize("acc", ["fp32", "fp16"])
def test_reference_fp16_harness_on_tcgemm(acc):
    env = {"PROFILE_SIZE": "1024"}
    if acc == "fp16":
        env["TCG_ACC"] = "fp16"
    out = _run("ref_main_fp16_on_tcgemm", env)
    m = re.search(r"\[verify\]\s+M=512 N=512 K=512\s+(PASS|FAIL)\s+max_abs=(\S+)", out)
    assert m and m.group(1) == "PASS", out
    # the reference's own kernels logged 2.3097e-07 (fp32 accumulation) and
    # 2.0949e-04 (fp16 accumulation) against its f32 CPU GEMM
    assert float(m.group(2)) < (1e-6 if acc == "fp32" else 2e-3), out
    assert "[profile] tcgemm_f16 | M=1024 N=1024 K=1024 B=4" in out, out
