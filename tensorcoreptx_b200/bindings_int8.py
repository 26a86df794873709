"""Module-level mirror of the reference's int8 extension (bindings/bindings_int8.cpp:36-39):
``from tensorcoreptx_b200 import bindings_int8; C = bindings_int8.gemm_int8(A, BT)``."""
from .gemm import gemm_int8  # noqa: F401
