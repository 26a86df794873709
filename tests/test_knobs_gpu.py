"""GPU parity under the library's tuning switches.

The environment switches are read once per process, so each configuration
runs in a child process: static round-robin scheduling instead of cluster
launch control (TCG_STATIC_SCHEDULE=1), plain stores instead of TMA stores
for C (TCG_TMA_STORE=0), no column-half tail split (TCG_TAIL_SPLIT=0), the
stream-K split of partial waves (TCG_STREAM_K=1).  Each
child multiplies multi-wave and single-wave int8 problems (bit-exact against
the oracle) and an fp16 problem (bit-identical to the default
configuration's result, which the parent computes), for every tile shape.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
import tensorcoreptx_b200 as T
from oracle import oracle as O

out_path = sys.argv[2]
dev = "cuda:0"
rng = np.random.default_rng(5)
results = {}
for (M, N, K) in ((3328, 3328, 256), (300, 520, 128), (4096, 3072, 512)):
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (N, K), dtype=np.int8)
    ref = O.gemm_s8(A, B, threads=8)
    At, Bt = torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev)
    for mode in (1, 2, 3, 4):
        T.set_cta_pair(mode)
        C = T.gemm_int8(At, Bt).cpu().numpy()
        assert np.array_equal(C, ref), ("int8", M, N, K, mode)
    T.set_cta_pair(0)
M = N = 2304
K = 192
Ah = rng.uniform(-1, 1, (M, K)).astype(np.float16)
Bh = rng.uniform(-1, 1, (K, N)).astype(np.float16)
A16, B16 = torch.from_numpy(Ah).to(dev), torch.from_numpy(Bh).to(dev)
for mode in (1, 2, 3, 4):
    T.set_cta_pair(mode)
    results[f"f16_{mode}"] = T.gemm_fp16(A16, B16).cpu().numpy()
T.set_cta_pair(0)
# 96 two-CTA 512 x 256 tiles on 74 pairs (fp16 keeps one k order per
# element: never split, whatever the switch)
Ah = rng.uniform(-1, 1, (4096, 512)).astype(np.float16)
Bh = rng.uniform(-1, 1, (512, 3072)).astype(np.float16)
A16, B16 = torch.from_numpy(Ah).to(dev), torch.from_numpy(Bh).to(dev)
for acc in ("fp32", "fp16"):
    results[f"f16_sk_{acc}"] = T.gemm_fp16(A16, B16, acc=acc).cpu().numpy()
assert T.check_device_error() == 0
np.savez(out_path, **results)
print("child ok")
"""


def _run(env_extra, tmp_path, name):
    env = dict(os.environ)
    env.update(env_extra)
    out = str(tmp_path / f"{name}.npz")
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT, out], env=env, cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return dict(np.load(out))


@pytest.fixture(scope="module")
def default_result(tmp_path_factory):
    return _run({}, tmp_path_factory.mktemp("knobs"), "default")


@pytest.mark.parametrize("env", [{"TCG_STATIC_SCHEDULE": "1"}, {"TCG_TMA_STORE": "0"},
                                 {"TCG_TAIL_SPLIT": "0"}, {"TCG_STREAM_K": "1"},
                                 {"TCG_STATIC_SCHEDULE": "1", "TCG_TAIL_SPLIT": "0", "TCG_TMA_STORE": "0"}],
                         ids=["static", "plain_stores", "no_tail_split", "stream_k", "all_off"])
def test_switch_keeps_results(env, default_result, tmp_path):
    res = _run(env, tmp_path, "switched")
    for key, ref in default_result.items():
        assert np.array_equal(res[key].view(np.uint32), ref.view(np.uint32)), key
