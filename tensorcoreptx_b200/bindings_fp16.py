"""Module-level mirror of the reference's fp16 extension (bindings/bindings_fp16.cpp:39-42):
``from tensorcoreptx_b200 import bindings_fp16; C = bindings_fp16.gemm_fp16(A, B)``."""
from .gemm import gemm_fp16  # noqa: F401
