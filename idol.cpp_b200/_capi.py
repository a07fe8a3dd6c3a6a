"""ctypes binding of libidol_b200.so (the C-ABI in include/idol_b200.h).

The library is the product: nothing here computes anything itself. If the shared library is missing or cannot be
loaded, every call raises ``LibraryMissing``; there is no fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libidol_b200.so"

OK, ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED, ERR_DEVICE = 0, 1, 2, 3, 4
F32, F16, BF16 = 0, 1, 2
ACT_NONE, ACT_GELU_ERF, ACT_GELU_TANH, ACT_SILU = 0, 1, 2, 3
EPI_BIAS_AFTER_ROUND = 0x1
GEMM_WHOLE_K = 0x2

# Every symbol include/idol_b200.h declares, with (restype, argtypes).
_vp, _i32, _i64, _u32p = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.POINTER(ctypes.c_uint)
SIGNATURES = {
    "idol_b200_last_error": (ctypes.c_char_p, []),
    "idol_b200_version": (_i32, []),
    "idol_b200_device_status": (_i32, [_i32, _u32p]),
    "idol_b200_q8_bytes": (_i64, [_i32, _i32]),
    "idol_b200_q8_tiled_bytes": (_i64, [_i32, _i32]),
    "idol_b200_q8_quantize": (_i32, [_vp, _i64, _i64, _vp, _vp]),
    "idol_b200_q8_repack": (_i32, [_vp, _i32, _i32, _vp, _vp]),
    "idol_b200_q4_0_bytes": (_i64, [_i32, _i32]),
    "idol_b200_q4_0_repack": (_i32, [_vp, _i32, _i32, _vp, _vp]),
    "idol_b200_q4_k_bytes": (_i64, [_i32, _i32]),
    "idol_b200_q4_k_tiled_bytes": (_i64, [_i32, _i32]),
    "idol_b200_q4_k_repack": (_i32, [_vp, _i32, _i32, _vp, _vp]),
    "idol_b200_q4_k_dequantize": (_i32, [_vp, _i32, _i32, _vp, _i32, _vp]),
    "idol_b200_q4_k_view": (_i32, [_vp, _vp, _i32, _i32, _i32, ctypes.POINTER(_vp)]),
    "idol_b200_q8_unpack": (_i32, [_vp, _i32, _i32, _vp, _vp]),
    "idol_b200_q8_dequantize": (_i32, [_vp, _i32, _i32, _vp, _i32, _vp]),
    "idol_b200_q8_upload": (_i32, [_vp, _i64, _i32, _i32, _vp, _i32, ctypes.POINTER(_vp)]),
    "idol_b200_q8_import": (_i32, [_vp, _i64, _i32, _i32, _vp, _i32, _vp, ctypes.POINTER(_vp)]),
    "idol_b200_q8_view": (_i32, [_vp, _vp, _i32, _i32, _i32, ctypes.POINTER(_vp)]),
    "idol_b200_q8_free": (_i32, [_vp]),
    "idol_b200_q8_info": (_i32, [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                                 ctypes.POINTER(_i64)]),
    "idol_b200_q8_export": (_i32, [_vp, _vp, _i64, _vp]),
    "idol_b200_q8_gemm": (_i32, [_vp, _vp, _i32, _i64, _i64, _i32, _i32, _vp, _i64, _i32, _i32, _vp, _i32, _i64,
                                 _vp]),
    "idol_b200_q8_gemm_heads": (_i32, [_vp, _vp, _i64, _i64, _vp, _i64, _i32, _i32, _vp, _vp, _vp]),
    "idol_b200_q8_gemm_int8act_workspace_bytes": (_i64, [_i64, _i32]),
    "idol_b200_q8_gemm_int8act": (_i32, [_vp, _vp, _i32, _i64, _i64, _i32, _i32, _vp, _i64, _i32, _vp, _i32, _i64,
                                         _vp, _i64, _vp]),
    "idol_b200_norm_rows": (_i32, [_vp, _i32, _i64, _i32, _i64, ctypes.c_float, _vp, _vp, _vp, _vp, _vp, _i32, _i64,
                                   _vp]),
    "idol_b200_rms_heads": (_i32, [_vp, _i32, _i64, _i64, _i32, _i32, _vp, _vp]),
    "idol_b200_attention": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i32, _i32, _vp, _i32, _i64, _i32, _vp]),
    "idol_b200_block_create": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, ctypes.c_float, ctypes.POINTER(_vp)]),
    "idol_b200_block_free": (_i32, [_vp]),
    "idol_b200_block_workspace_bytes": (_i64, [_vp, _i64]),
    "idol_b200_block_forward": (_i32, [_vp, _vp, _i32, _i64, _i32, _vp, _i64, _vp]),
    "idol_b200_gs_block_create": (_i32, [_vp] * 14 + [_i32, _i32, ctypes.c_float, ctypes.POINTER(_vp)]),
    "idol_b200_gs_block_free": (_i32, [_vp]),
    "idol_b200_gs_block_workspace_bytes": (_i64, [_vp, _i64, _i64]),
    "idol_b200_gs_block_forward": (_i32, [_vp, _vp, _i32, _i64, _i32, _vp, _i64, _vp, _i64, _vp]),
    "idol_b200_gs_decoder_create": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp, ctypes.c_float, _vp,
                                            ctypes.POINTER(_vp)]),
    "idol_b200_gs_decoder_free": (_i32, [_vp]),
    "idol_b200_gs_decoder_workspace_bytes": (_i64, [_vp, _i64, _i64]),
    "idol_b200_gs_decoder_features": (_i32, [_vp, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp]),
    "idol_b200_gs_to_gaussians": (_i32, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "idol_b200_oct_block_create": (_i32, [_vp] * 8 + [_i32, _i32, ctypes.POINTER(_vp)]),
    "idol_b200_oct_block_free": (_i32, [_vp]),
    "idol_b200_oct_decoder_create": (_i32, [_vp, _i32] + [_vp] * 8 + [_i32, _vp, _i32, ctypes.c_float,
                                                                         ctypes.POINTER(_vp)]),
    "idol_b200_oct_decoder_free": (_i32, [_vp]),
    "idol_b200_oct_decoder_workspace_bytes": (_i64, [_vp, _i64, _i64]),
    "idol_b200_oct_logits": (_i32, [_vp, _vp, _i64, ctypes.c_float, _vp, _i64, _vp, _vp, _i64, _vp]),
    "idol_b200_oct_sample_anchors": (_i32, [_vp, _vp, _i64, _i32, _i32, ctypes.c_uint64, _vp, _vp, _i64, _vp]),
    "idol_b200_oct_sampler_create": (_i32, [_i32, _i32, ctypes.c_uint64, ctypes.POINTER(_vp)]),
    "idol_b200_oct_sampler_free": (_i32, [_vp]),
    "idol_b200_oct_sampler_cells": (_i32, [_vp, ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_float)]),
    "idol_b200_oct_sampler_centres": (_i32, [_vp, _vp]),
    "idol_b200_oct_sampler_step": (_i32, [_vp, _vp]),
    "idol_b200_oct_sampler_points": (_i32, [_vp, _vp]),
    "idol_b200_gaussian_mlp_create": (_i32, [_vp, _vp, _vp, ctypes.POINTER(_vp)]),
    "idol_b200_gaussian_mlp_free": (_i32, [_vp]),
    "idol_b200_gaussian_mlp_workspace_bytes": (_i64, [_vp, _i64]),
    "idol_b200_gaussian_mlp_forward": (_i32, [_vp, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp]),
    "idol_b200_gaussian_mlp_forward_static": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp, _vp]),
    "idol_b200_gaussian_heads": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp]),
}


class LibraryMissing(RuntimeError):
    pass


class IdolError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"idol_b200 error {code}: {msg}")
        self.code = code


_lib = None


def lib():
    """The loaded library with argument types set. Raises LibraryMissing when it is not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise LibraryMissing(f"{LIB_PATH} is not built: run `python idol.cpp_b200/build.py` (nvcc, sm_100a)")
        try:
            L = ctypes.CDLL(str(LIB_PATH))
        except OSError as exc:
            raise LibraryMissing(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    """Raise for a non-zero status: ValueError for invalid arguments (the reference's ValueError/invalid_argument),
    IdolError otherwise."""
    if rc == OK:
        return
    msg = (lib().idol_b200_last_error() or b"").decode(errors="replace")
    if rc == ERR_INVALID:
        raise ValueError(msg)
    raise IdolError(rc, msg)


def device_status(device: int) -> int:
    flags = ctypes.c_uint(0)
    check(lib().idol_b200_device_status(device, ctypes.byref(flags)))
    return int(flags.value)
