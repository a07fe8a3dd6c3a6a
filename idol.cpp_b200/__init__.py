"""idol.cpp_b200 - B200-native (sm_100a) Q8_0 linear hot path of idol.cpp.

Host-side mirror of the reference's operator boundary for that path. The arithmetic lives in libidol_b200.so (CUDA,
built by build.py), reached through its C-ABI (include/idol_b200.h) from ``_capi``. The directory name is not a
Python identifier, so callers load it under the name ``idol_b200`` (see ``__graft_entry__.load_package``).
"""
from . import _capi
from .q8 import (PackedLinear, dequantize_tiled, enable_fused_packed, fused_linear, gemm_into, q4_0_bytes, q4_k_bytes,
                 q4_k_tiled_bytes, q8_bytes, q8_linear, quantize, repack, repack_q4_0, repack_q4_k, tiled_bytes,
                 unpack)

__all__ = ["_capi", "PackedLinear", "dequantize_tiled", "enable_fused_packed", "fused_linear", "gemm_into",
           "q4_0_bytes", "q4_k_bytes", "q4_k_tiled_bytes", "q8_bytes", "q8_linear", "quantize", "repack", "repack_q4_0",
           "repack_q4_k", "tiled_bytes", "unpack"]
