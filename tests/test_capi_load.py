"""The C-ABI library loads on a machine without a GPU and exports every symbol include/idol_b200.h declares (no
compute calls here); host-side argument checks answer with status codes, not crashes."""
import ctypes
import re

from conftest import ROOT


def _declared():
    text = (ROOT / "include" / "idol_b200.h").read_text()
    return sorted(set(re.findall(r"\b(idol_b200_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = _declared()
    for needed in ("idol_b200_q8_gemm", "idol_b200_q8_upload", "idol_b200_q8_quantize", "idol_b200_q8_repack",
                   "idol_b200_q8_unpack", "idol_b200_last_error"):
        assert needed in names


def test_library_exports_every_declared_symbol(pkg):
    L = pkg._capi.lib()
    missing = [n for n in _declared() if not hasattr(L, n)]
    assert not missing, missing
    assert set(pkg._capi.SIGNATURES) == set(_declared())


def test_sizes_and_argument_errors_without_a_device(pkg):
    L = pkg._capi.lib()
    assert L.idol_b200_q8_bytes(4096, 1024) == 4096 * 32 * 34
    assert L.idol_b200_q8_tiled_bytes(14, 128) == 1 * 2 * 8704
    assert L.idol_b200_q8_tiled_bytes(300, 96) == 3 * 2 * 8704
    assert L.idol_b200_q8_bytes(16, 33) == -1
    h = ctypes.c_void_p()
    assert L.idol_b200_q8_upload(None, 0, 16, 48, None, 0, ctypes.byref(h)) == pkg._capi.ERR_INVALID
    assert b"multiple of 32" in L.idol_b200_last_error()
    assert L.idol_b200_q8_view(None, None, 16, 64, 0, ctypes.byref(h)) == pkg._capi.ERR_INVALID
    assert L.idol_b200_q8_gemm(None, None, 2, 1, 64, 0, 16, None, 0, 0, 0, None, 2, 16, None) == pkg._capi.ERR_INVALID
    assert L.idol_b200_version() >= 100


def test_fused_linear_rejects_what_the_reference_rejects(pkg):
    import pytest
    import torch
    x = torch.zeros(2, 64, dtype=torch.bfloat16)
    packed = torch.zeros(16 * 2 * 34, dtype=torch.uint8)
    with pytest.raises(ValueError, match="unsupported fused linear input"):
        pkg.fused_linear(x, packed, (16, 64), 8)
