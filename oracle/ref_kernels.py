"""Run the reference's own GPU kernels, recompiled unchanged for sm_100a into
oracle/_ref/libref_<kernel>.so (``make -C oracle ref``), on torch tensors.

Test / baseline infrastructure only: the GPU tests compare against these
kernels, and bench.py reports their speed as a baseline (outside its timed
region).  Each library exposes
``int ref_launch(A, B, C, M, N, K, batches, stream)`` around the kernel file's
``launch_kernel`` (oracle/ref_kernel_shim.cu).  The reference kernels need
M % 32 == 0, N % 64 == 0 and K a multiple of their K tile (they do not
bounds-check), so callers only use such shapes.
"""
import ctypes as C
import os

REF_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")

KERNELS = {
    "fp16_wmma": "fp16", "fp16_ptx_fp16acc": "fp16",
    "int8_wmma": "int8", "int8_ptx_mma_k32": "int8",
    "int4_wmma": "int4", "int4_ptx_mma_k64_x4_x2nontrans_ca": "int4",
    "int4_ptx_mma_k64_x2_x2nontrans_ca": "int4",
}
K_TILE = {"fp16_wmma": 16, "fp16_ptx_fp16acc": 16, "int8_wmma": 16, "int8_ptx_mma_k32": 32,
          "int4_wmma": 32, "int4_ptx_mma_k64_x4_x2nontrans_ca": 64, "int4_ptx_mma_k64_x2_x2nontrans_ca": 64}

_libs = {}


def available(name):
    return os.path.exists(os.path.join(REF_DIR, f"libref_{name}.so"))


def lib(name):
    if name not in _libs:
        L = C.CDLL(os.path.join(REF_DIR, f"libref_{name}.so"), mode=os.RTLD_LOCAL | os.RTLD_NOW)
        L.ref_launch.restype = C.c_int
        L.ref_launch.argtypes = [C.c_void_p] * 3 + [C.c_int] * 4 + [C.c_void_p]
        _libs[name] = L
    return _libs[name]


def shape_ok(name, M, N, K):
    return M % 32 == 0 and N % 64 == 0 and K % K_TILE[name] == 0


def run(name, A, B, M, N, K, batches=1):
    """C = A x B with the reference kernel `name`; A/B torch CUDA tensors in
    the reference layouts (fp16: B is K x N; int8/int4: B is BT)."""
    import torch
    assert shape_ok(name, M, N, K), (name, M, N, K)
    dt = torch.float32 if KERNELS[name] == "fp16" else torch.int32
    Cm = torch.zeros((batches, M, N) if batches > 1 else (M, N), dtype=dt, device=A.device)
    rc = lib(name).ref_launch(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), M, N, K, batches,
                              torch.cuda.current_stream(A.device).cuda_stream)
    if rc != 0:
        raise RuntimeError(f"reference kernel {name} launch failed: cuda error {rc}")
    return Cm
