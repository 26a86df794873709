"""Stream-K (integer kinds, opt-in with TCG_STREAM_K=1): problems of one to
four waves of two-CTA 512 x 256 tiles with a partial last wave are split so
every resident pair takes an equal share of the tiles' k-blocks; a tile cut
between two pairs is stored by the first (its partial sums, flagged) and
completed by the second with TMA reduce-add stores.  The switch is read once
per process, so the checks run in a child process: exact against a float64
GEMM (exact below 2^53) with ragged edges, batches, repeated launches (the
hand-off flags are reused), CUDA-graph replays (same tag each replay), int4,
and the dequantising epilogue (not split: it rounds per element)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys
import torch
sys.path.insert(0, sys.argv[1])
import tensorcoreptx_b200 as T

DEV = "cuda:0"


def exact_int(A, BT):
    # A x BT^T in float64: every partial sum is an integer below 2^53
    return (A.double() @ BT.double().t()).round().to(torch.int64)


for (M, N, K) in ((4096, 4096, 1024), (4000, 3900, 2048), (4096, 3072, 512), (2560, 8192, 768)):
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    A = torch.randint(-128, 128, (M, K), generator=g, device=DEV, dtype=torch.int8)
    BT = torch.randint(-128, 128, (N, K), generator=g, device=DEV, dtype=torch.int8)
    C = T.gemm_int8(A, BT)
    assert T.last_tile_m() == 512
    assert torch.equal(C.to(torch.int64), exact_int(A, BT)), (M, N, K)

# batches fold into the split; back-to-back launches reuse the flags
g = torch.Generator(device=DEV).manual_seed(3)
A = torch.randint(-128, 128, (2, 2048, 1024), generator=g, device=DEV, dtype=torch.int8)
BT = torch.randint(-128, 128, (2, 4096, 1024), generator=g, device=DEV, dtype=torch.int8)
ref = torch.stack([exact_int(A[b], BT[b]) for b in range(2)])
for _ in range(5):
    assert torch.equal(T.gemm_int8(A, BT).to(torch.int64), ref), "batched"

# a CUDA graph replays the same tag; the tail resets a flag it consumes
A = torch.randint(-128, 128, (4096, 1024), generator=g, device=DEV, dtype=torch.int8)
BT = torch.randint(-128, 128, (4096, 1024), generator=g, device=DEV, dtype=torch.int8)
ref = exact_int(A, BT)
s = torch.cuda.Stream()
with torch.cuda.stream(s):
    C = T.gemm_int8(A, BT)
s.synchronize()
graph = torch.cuda.CUDAGraph()
with torch.cuda.graph(graph, stream=s):
    C = T.gemm_int8(A, BT)
for _ in range(4):
    C.fill_(0)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(C.to(torch.int64), ref), "graph"
del graph

# int4 (split) and the dequantising epilogue (not split)
n, k = 4096, 1024
qa = torch.randint(-127, 128, (n, k), generator=g, device=DEV, dtype=torch.int8)
qb = torch.randint(-127, 128, (n, k), generator=g, device=DEV, dtype=torch.int8)
sa = torch.tensor([0.0123], device=DEV)
sb = torch.tensor([0.0456], device=DEV)
assert torch.equal(T.gemm_int8_dequant(qa, qb, sa, sb), T.gemm_int8(qa, qb).float() * (sa * sb)), "dequant"
Ap = torch.randint(-128, 128, (n, k // 2), generator=g, device=DEV, dtype=torch.int8)
Bp = torch.randint(-128, 128, (n, k // 2), generator=g, device=DEV, dtype=torch.int8)
assert torch.equal(T.gemm_int4(Ap, Bp), T.gemm_int8(T.unpack_int4(Ap), T.unpack_int4(Bp))), "int4"
assert T.check_device_error() == 0
print("child ok")
"""


def test_stream_k_exact_in_child():
    env = dict(os.environ)
    env["TCG_STREAM_K"] = "1"
    env["TCG_DEBUG"] = "1"
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], env=env, cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "child ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
    assert "stream-k" in r.stderr  # the split was taken
