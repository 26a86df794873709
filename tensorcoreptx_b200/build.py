"""In-tree build of the native libraries (nvcc, sm_100a only).

    python -m tensorcoreptx_b200.build          # build what is out of date
    python -m tensorcoreptx_b200.build --force  # rebuild everything

Outputs, next to this file:
    libtcgemm.so                 the C ABI of include/tcgemm.h (all kernels)
    libtcgemm_compat_f16.so      reference-compatible C++ `launch_kernel` +
    libtcgemm_compat_s8.so       `Solver*` per precision (include/tcgemm_compat.h),
    libtcgemm_compat_s4.so       one per precision as the reference links one
                                 kernel file per binary
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
                 "-I" + INCLUDE]

LIB = os.path.join(HERE, "libtcgemm.so")
COMPAT = {p: os.path.join(HERE, f"libtcgemm_compat_{p}.so") for p in ("f16", "s8", "s4")}


def _sources(*names):
    return [os.path.join(CSRC, n) for n in names]


def _deps():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + \
        [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def build(force: bool = False, verbose: bool = True) -> list[str]:
    deps = _deps()
    built = []
    if force or _stale(LIB, deps):
        _run([NVCC] + COMMON + _sources("tcgemm.cu") + ["-o", LIB], verbose)
        built.append(LIB)
    defines = {"f16": "TCG_COMPAT_F16", "s8": "TCG_COMPAT_S8", "s4": "TCG_COMPAT_S4"}
    for prec, out in COMPAT.items():
        if force or _stale(out, deps + [LIB]):
            _run([NVCC] + COMMON + ["-D" + defines[prec]] + _sources("compat.cu") +
                 ["-L" + HERE, "-ltcgemm", "-Xlinker", "-rpath=$ORIGIN", "-o", out], verbose)
            built.append(out)
    return built


if __name__ == "__main__":
    build(force="--force" in sys.argv)
