"""Generate the golden fixtures in tests/golden/ from the reference's own code.

The reference's host code (src/data.cu, src/data_int8.cu, src/data_int4.cu of
MattJBorowski1991/TensorCorePTX) is compiled unchanged into oracle/_ref/ by
``make -C oracle ref``.  This script runs *that* code -- its seeded generators
and naive CPU GEMMs -- and stores the inputs and outputs as small .npz files,
so the oracle restatement can be pinned on machines that do not have the
reference tree.  Known answers printed by the reference in its committed
Nsight logs are stored in known_answers.json (copied by hand, with sources).

Run:  make -C oracle all ref && python tests/golden/make_golden.py
"""
import ctypes as C
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

# (M, N, K) cases: the reference's verify size is 512^3; these small ones keep
# the fixtures a few tens of KB while covering non-square and ragged shapes.
CASES = [(64, 64, 64), (96, 80, 128), (32, 64, 256)]


def vp(a):
    return a.ctypes.data_as(C.c_void_p)


def main():
    out = {}
    for prec in ("int8", "int4", "fp16"):
        L = O.ref_data_lib(prec)
        if L is None:
            raise SystemExit("oracle/_ref missing: run `make -C oracle ref` first")
        for (M, N, K) in CASES:
            if prec == "int8":
                A = np.empty(M * K, np.int8)
                B = np.empty(N * K, np.int8)
                Cm = np.zeros(M * N, np.int32)
            elif prec == "int4":
                A = np.empty(M * K // 2, np.int8)
                B = np.empty(N * K // 2, np.int8)
                Cm = np.zeros(M * N, np.int32)
            else:
                A = np.empty(M * K, np.uint16)
                B = np.empty(K * N, np.uint16)
                Cm = np.zeros(M * N, np.float32)
            L.gen(vp(A), vp(B), M, N, K, 1)
            L.gemm(vp(A), vp(B), vp(Cm), M, N, K)
            key = f"{prec}_{M}x{N}x{K}"
            np.savez_compressed(os.path.join(HERE, key + ".npz"), A=A, B=B, C=Cm,
                                shape=np.array([M, N, K]))
            out[key] = {"M": M, "N": N, "K": K}
    # a 512^3 int8 / int4 row of C (row 304 covers the negative-control cell)
    for prec in ("int8", "int4"):
        L = O.ref_data_lib(prec)
        M = N = K = 512
        kb = K if prec == "int8" else K // 2
        A = np.empty(M * kb, np.int8)
        B = np.empty(N * kb, np.int8)
        L.gen(vp(A), vp(B), M, N, K, 1)
        rows = np.zeros((2, N), np.int32)
        for i, r in enumerate((0, 304)):
            L.gemm(C.c_void_p(A.ctypes.data + r * kb), vp(B), vp(rows[i]), 1, N, K)
        np.savez_compressed(os.path.join(HERE, f"{prec}_512_rows.npz"), rows=rows,
                            row_ids=np.array([0, 304]))
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print("wrote", len(out), "cases")


if __name__ == "__main__":
    main()
