"""int4 counterpart of bindings_int8 (the reference has no int4 binding; its int4
path is src/main_int4.cu): ``bindings_int4.gemm_int4(A_packed, BT_packed)``."""
from .gemm import gemm_int4  # noqa: F401
