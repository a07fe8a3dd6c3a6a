"""GGUF Q4_K (fused_linear kind 44) through the Q4_K tiled layout.

CPU: the oracle's Q4_K decoder equals gguf-py 0.19.0's dequantize and the reference's own expansion
(tools/idol_packed.py PackedLinear.dequantize) on the committed golden vectors, exactly, and so does PackedLinear's
CPU expansion here; the C-ABI sizes and argument checks answer without a GPU.
GPU: the device repack dequantises to exactly those fp32 weights (and to their bf16 / fp16 roundings); fused_linear
(kind 44) and PackedLinear(Q4_K) on every tile width, split and the streaming small-M kernel meet the bars of the
other kinds: max |y - ref| <= 2e-2 x rms(ref) plus the output's rounding, and the reference's relative Frobenius bar
(< 1e-3, tests/python/test_fused_packed.py:52-59), against a float64 product of the same bf16 weights.
"""
import types

import numpy as np
import pytest
import torch

from conftest import GOLDEN

Q4K = 12  # gguf.GGMLQuantizationType.Q4_K


def _golden():
    z = np.load(GOLDEN / "q4_k.npz")
    return int(z["rows"]), int(z["cols"]), z["q4k"], z["gguf_dequant"], z["ref_dequant"]


def _random_q4k(rows, cols, seed):
    """Seeded Q4_K super-blocks: fp16 d and dmin of weight-like size, random scale / min bytes and codes."""
    rng = np.random.default_rng(seed)
    nsb = cols // 256
    blocks = rng.integers(0, 256, size=(rows, nsb, 144), dtype=np.uint8)
    blocks[:, :, 0:2] = np.abs(rng.normal(0, 4e-3, (rows, nsb))).astype(np.float16).view(np.uint8).reshape(
        rows, nsb, 2)
    blocks[:, :, 2:4] = np.abs(rng.normal(0, 2e-2, (rows, nsb))).astype(np.float16).view(np.uint8).reshape(
        rows, nsb, 2)
    return blocks.reshape(-1)


def _source(q4k, rows, cols):
    return types.SimpleNamespace(shape=np.array([cols, rows]), tensor_type=Q4K, data=q4k)


def test_oracle_decoder_is_exact(oracle):
    rows, cols, q4k, deq, ref_deq = _golden()
    mine = oracle.q4_k_dequantize(q4k, rows, cols)
    assert np.array_equal(mine, deq) and np.array_equal(mine, ref_deq)


def test_packed_linear_cpu_expansion_is_exact(pkg):
    rows, cols, q4k, deq, _ = _golden()
    layer = pkg.PackedLinear(_source(q4k, rows, cols), None)
    assert np.array_equal(layer.dequantize(torch.float32).numpy(), deq)
    assert torch.equal(layer.dequantize(torch.bfloat16), torch.from_numpy(deq).to(torch.bfloat16))


def test_capi_sizes_and_errors(pkg):
    L = pkg._capi.lib()
    assert L.idol_b200_q4_k_bytes(4096, 1024) == 4096 * 4 * 144
    assert L.idol_b200_q4_k_bytes(16, 96) == -1
    assert L.idol_b200_q4_k_tiled_bytes(200, 768) == 2 * 12 * 6144
    assert L.idol_b200_q4_k_repack(None, 16, 256, None, None) == pkg._capi.ERR_INVALID
    assert b"NULL" in L.idol_b200_last_error()
    h = pkg._capi.ctypes.c_void_p()
    assert L.idol_b200_q4_k_view(None, None, 16, 96, 0, pkg._capi.ctypes.byref(h)) == pkg._capi.ERR_INVALID
    assert b"multiple of 256" in L.idol_b200_last_error()


@pytest.mark.gpu
def test_device_repack_dequantises_exactly(pkg, cuda):
    rows, cols, q4k, deq, _ = _golden()
    tiles = pkg.repack_q4_k(torch.from_numpy(q4k).to(cuda), rows, cols)
    assert tiles.numel() == pkg.q4_k_tiled_bytes(rows, cols)
    assert np.array_equal(pkg.dequantize_tiled(tiles, rows, cols, torch.float32).cpu().numpy(), deq)
    for dt in (torch.bfloat16, torch.float16):
        got = pkg.dequantize_tiled(tiles, rows, cols, dt).cpu()
        assert torch.equal(got, torch.from_numpy(deq).to(dt)), dt


def _reference(x, w_deq, bias, dtype):
    """fused_linear's semantics with a float64 product: X . bf16/fp16(W)^T rounded to the output dtype, then + bias in
    that dtype (tools/idol_triton.py:84-89)."""
    wq = torch.from_numpy(w_deq).to(dtype).double()
    y = (x.double().cpu() @ wq.T).to(dtype)
    if bias is not None:
        y = (y.float() + bias.float().cpu()).to(dtype)
    return y.double().numpy()


def _bars(y, ref, dtype, what):
    y = y.float().cpu().double().numpy()
    rms = np.sqrt((ref ** 2).mean())
    half_ulp = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    excess = (np.abs(y - ref) - half_ulp * np.abs(ref)).max()
    assert excess <= 2e-2 * rms, f"{what}: {excess:.3e} > 2e-2 x rms {rms:.3e}"
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel < 1e-3, f"{what}: relative Frobenius error {rel:.2e}"


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 3072, 1024), (16, 200, 768), (7, 300, 4096), (300, 71, 256),
                                   (64, 512, 2048), (4097, 1024, 1024), (16384, 1024, 1024)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_linear_q4_k(pkg, oracle, cuda, m, n, k, dtype):
    """Decode sizes (the streaming kernel, K split across a cluster at 4096), split-K, and the tcgen05 kernel."""
    q4k = _random_q4k(n, k, m + n + k)
    w_deq = oracle.q4_k_dequantize(q4k, n, k)
    g = torch.Generator(device=cuda).manual_seed(m * 3 + k)
    x = torch.randn((m, k), device=cuda, generator=g).to(dtype)
    bias = (torch.randn(n, device=cuda, generator=g) * 0.1).to(dtype)
    packed = torch.from_numpy(q4k).to(cuda)
    y = pkg.fused_linear(x, packed, (n, k), 44, bias)
    torch.cuda.synchronize()
    assert y.shape == (m, n) and y.dtype == dtype
    rows = np.unique(np.linspace(0, m - 1, min(m, 64)).astype(int))
    ref = _reference(x[torch.from_numpy(rows).to(cuda)], w_deq, bias, dtype)
    _bars(y[torch.from_numpy(rows).to(cuda)], ref, dtype, f"Q4_K {m}x{n}x{k} {dtype}")


@pytest.mark.gpu
@pytest.mark.parametrize("bn", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("splits", [1, 2, 4])
def test_every_tile_width_and_split_q4_k(pkg, oracle, cuda, bn, splits, monkeypatch):
    monkeypatch.setenv("IDOL_B200_GEMM_BN", str(bn))
    monkeypatch.setenv("IDOL_B200_GEMM_SPLITS", str(splits))
    monkeypatch.setenv("IDOL_B200_GEMV", "0")
    m, n, k = 300, 200, 1024
    q4k = _random_q4k(n, k, bn * 10 + splits)
    w_deq = oracle.q4_k_dequantize(q4k, n, k)
    g = torch.Generator(device=cuda).manual_seed(bn + splits)
    x = torch.randn((m, k), device=cuda, generator=g).to(torch.bfloat16)
    tiles = pkg.repack_q4_k(torch.from_numpy(q4k).to(cuda), n, k)
    y = torch.empty((m, n), device=cuda, dtype=torch.float32)
    pkg.gemm_into(y, x, tiles, None, n, k)
    torch.cuda.synchronize()
    ref = x.double().cpu() @ torch.from_numpy(w_deq).to(torch.bfloat16).double().T
    err = (y.double().cpu() - ref).abs().max().item()
    rms = ref.pow(2).mean().sqrt().item()
    assert err <= 2e-2 * rms, f"bn={bn} splits={splits}: {err:.3e} > 2e-2 x {rms:.3e}"


@pytest.mark.gpu
def test_packed_linear_q4_k_fused_and_expanded(pkg, oracle, cuda):
    n, k, m = 384, 512, 100
    q4k = _random_q4k(n, k, 9)
    bias = (torch.randn(n) * 0.1).to(torch.bfloat16)  # the reference wants the bias in the activation dtype
    layer = pkg.PackedLinear(_source(q4k, n, k), bias).to(cuda)
    x = torch.randn((2, m, k), device=cuda).to(torch.bfloat16)
    with torch.no_grad():
        expanded = layer(x)  # not fused: dequantize (device kernel) + F.linear
        assert pkg.enable_fused_packed(layer) == 1
        fused = layer(x)
    torch.cuda.synchronize()
    assert fused.shape == expanded.shape == (2, m, n)
    dense = layer.dequantize(torch.bfloat16)
    reference = (x.float() @ dense.float().T).to(torch.bfloat16) + layer.bias  # round, then add the bias
    rel = ((fused.float() - reference.float()).norm() / reference.float().norm()).item()
    assert rel < 1e-3, rel
    # The expansion path is F.linear (cuBLAS adds the bias before its one rounding): within two bf16 roundings.
    rel = ((expanded.float() - reference.float()).norm() / reference.float().norm()).item()
    assert rel < 4e-3, rel
    w_deq = oracle.q4_k_dequantize(q4k, n, k)
    assert torch.equal(layer.dequantize(torch.float32).cpu(), torch.from_numpy(w_deq))
