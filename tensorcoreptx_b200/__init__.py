"""tensorcoreptx_b200 -- B200-native (sm_100a) tensor-core GEMM library.

Drop-in for the GEMM hot path of MattJBorowski1991/TensorCorePTX:
fp16 (fp32 or fp16 accumulation), int8 and packed int4 GEMM on tcgen05
tensor cores, behind the reference's entry points:

* Python: ``gemm_fp16(A, B)``, ``gemm_int8(A, BT)`` (bindings/bindings_*.cpp)
  plus ``gemm_int4``;
* C ABI: include/tcgemm.h (libtcgemm.so);
* C++: ``launch_kernel`` / ``Solver*`` (include/tcgemm_compat.h,
  libtcgemm_compat_{f16,s8,s4}.so).
"""
from .host_gemm import gemm_fp16_host, gemm_int8_host
from .gemm import (check_device_error, gemm_fp8, gemm_int4_dequant, gemm_int8_dequant, quantize_absmax_int4,
                   quantize_absmax_int8, gemm_fp16, gemm_fp16_nk, gemm_int4, gemm_int8,
                   gemm_int8_kn, int4_workspace_size, last_tile_m, last_tile_n, set_cta_pair,
                   set_tile_n, unpack_int4)

__all__ = ["gemm_fp16", "gemm_fp16_nk", "gemm_int8", "gemm_int8_kn", "gemm_int4",
           "int4_workspace_size", "unpack_int4", "check_device_error", "set_tile_n",
           "last_tile_n", "last_tile_m", "set_cta_pair", "gemm_int8_host", "gemm_fp16_host",
           "quantize_absmax_int8", "quantize_absmax_int4", "gemm_int8_dequant", "gemm_int4_dequant",
           "gemm_fp8"]
