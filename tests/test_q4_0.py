"""GGUF Q4_0 (fused_linear kind 4) through the tiled Q8_0 layout.

CPU: the oracle's Q4_0 decoder equals gguf-py 0.19.0's dequantize and the reference's own expansion
(tools/idol_packed.py PackedLinear.dequantize) on the committed golden vectors, exactly; its Q4_0 -> Q8_0 conversion
keeps every weight; the C-ABI sizes and argument checks answer without a GPU.
GPU: the device conversion dequantises to exactly gguf's weights; fused_linear(kind 4) and PackedLinear(Q4_0) meet
the same bars as Q8_0 (max |y - ref| <= 2e-2 x rms against the fp32 oracle GEMM, and the reference's relative
Frobenius bar < 1e-3, tests/python/test_fused_packed.py:52-59).
"""
import ctypes
import types

import numpy as np
import pytest
import torch

from conftest import GOLDEN


def _golden():
    z = np.load(GOLDEN / "q4_0.npz")
    return z["w"].shape, z["q4"], z["gguf_dequant"], z["ref_dequant"]


def test_oracle_decoder_is_exact(oracle):
    (rows, cols), q4, deq, ref_deq = _golden()
    mine = oracle.q4_0_dequantize(q4, rows, cols)
    assert np.array_equal(mine, deq) and np.array_equal(mine, ref_deq)
    q8 = oracle.q4_0_to_q8(q4, rows, cols)
    assert np.array_equal(oracle.q8_dequantize(q8, rows, cols), deq)


def test_capi_sizes_and_errors(pkg):
    L = pkg._capi.lib()
    assert L.idol_b200_q4_0_bytes(4096, 1024) == 4096 * 32 * 18
    assert L.idol_b200_q4_0_bytes(16, 33) == -1
    assert L.idol_b200_q4_0_repack(None, 16, 64, None, None) == pkg._capi.ERR_INVALID
    assert b"NULL" in L.idol_b200_last_error()


@pytest.mark.gpu
def test_device_conversion_dequantises_exactly(pkg, cuda):
    (rows, cols), q4, deq, _ = _golden()
    tiles = pkg.repack_q4_0(torch.from_numpy(q4).to(cuda), rows, cols)
    got = pkg.dequantize_tiled(tiles, rows, cols, torch.float32).cpu().numpy()
    assert np.array_equal(got, deq)


def _q4(w):
    import gguf
    return np.asarray(gguf.quantize(np.ascontiguousarray(w, np.float32), gguf.GGMLQuantizationType.Q4_0),
                      dtype=np.uint8).reshape(-1)


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 3072, 1024), (16, 200, 96), (300, 71, 256), (4097, 1024, 1024)])
def test_fused_linear_q4_0_against_the_oracle(pkg, oracle, cuda, m, n, k):
    pytest.importorskip("gguf")
    rng = np.random.default_rng(m + n + k)
    w = rng.normal(0, 0.25, (n, k)).astype(np.float32)
    q4 = _q4(w)
    x = oracle.f32_to_bf16_round(rng.normal(0, 1, (m, k)).astype(np.float32))
    out = pkg.fused_linear(torch.from_numpy(x).to(cuda, torch.bfloat16), torch.from_numpy(q4).to(cuda), (n, k), 4)
    rows = np.unique(np.linspace(0, m - 1, min(m, 48)).astype(int))
    ref = oracle.gemm_q8(x[rows], oracle.q4_0_to_q8(q4, n, k), np.zeros(n, np.float32), n, k)
    y = out.float().cpu().numpy()[rows]
    rms = np.sqrt((ref.astype(np.float64) ** 2).mean())
    assert np.isfinite(y).all() and np.abs(y - ref).max() <= 2e-2 * rms


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_packed_linear_q4_0_meets_the_reference_bar(pkg, cuda, dtype):
    pytest.importorskip("gguf")
    rng = np.random.default_rng(4)
    for rows, columns, width in [(1, 7, 256), (41, 71, 256), (4097, 1024, 1024)]:
        data = _q4(rng.normal(0, 0.25, (columns, width)).astype(np.float32))
        tensor = types.SimpleNamespace(shape=np.array([width, columns]), tensor_type=2, data=data)
        layer = pkg.PackedLinear(tensor, None).to(cuda)
        value = torch.randn(rows, width * 2, device=cuda, dtype=dtype)[:, ::2]
        for bias in (None, torch.randn(columns, device=cuda, dtype=dtype)):
            output = pkg.fused_linear(value, layer.packed, layer.shape, 4, bias)
            layer.bias = torch.nn.Parameter(bias, requires_grad=False) if bias is not None else None
            layer.fused = False
            dense = layer.dequantize(dtype)
            assert torch.equal(dense.cpu(), layer.cpu().dequantize(dtype))  # device and host expansions agree
            layer.to(cuda)
            assert pkg.enable_fused_packed(layer) == 1
            torch.testing.assert_close(layer(value), output, rtol=0, atol=0)
            reference = (value.float() @ dense.float().T).to(dtype)
            if bias is not None:
                reference = reference + bias
            relative = (output.float() - reference.float()).norm() / reference.float().norm().clamp_min(1e-12)
            assert torch.isfinite(output).all() and relative < 1e-3, (rows, columns, width, float(relative))


@pytest.mark.gpu
def test_fused_linear_keeps_the_references_argument_errors(pkg, cuda):
    """Wrong byte counts and a K that is not a multiple of the kind's group raise ValueError for every kind."""
    x = torch.zeros(2, 256, device=cuda, dtype=torch.bfloat16)
    for kind, size in ((8, 16 * 8 * 34), (4, 16 * 8 * 18), (44, 16 * 144)):
        with pytest.raises(ValueError, match="invalid packed linear dimensions"):
            pkg.fused_linear(x, torch.zeros(size + 1, dtype=torch.uint8, device=cuda), (16, 256), kind)
    with pytest.raises(ValueError, match="invalid packed linear dimensions"):
        pkg.fused_linear(torch.zeros(2, 96, device=cuda, dtype=torch.bfloat16),
                         torch.zeros(16 * 144, dtype=torch.uint8, device=cuda), (16, 96), 44)
    with pytest.raises(ValueError, match="unsupported fused linear input"):
        pkg.fused_linear(x, torch.zeros(16 * 8 * 34, dtype=torch.uint8, device=cuda), (16, 256), 6)
