"""The CPU oracle is pinned before it is trusted: against gguf-py's bytes and the reference's own outputs, stored as
golden vectors (tests/golden/make_golden.py), and against the reference library itself when it was built here."""
import numpy as np
import pytest

from conftest import GOLDEN


def _gemm_cases():
    z = np.load(GOLDEN / "gemm.npz")
    names = sorted({k.split("/")[0] for k in z.files})
    return {n: {k.split("/")[1]: z[k] for k in z.files if k.startswith(n + "/")} for n in names}


def test_f16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.normal(0, s, 4000).astype(np.float32) for s in (1e-8, 1e-6, 1e-4, 1e-2, 1, 1e3, 6e4)])
    vals = np.concatenate([vals, np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e9, 2 ** -25, 2 ** -24, 3 * 2 ** -26,
                                           np.inf, -np.inf], np.float32)])
    mine = np.array([oracle.lib().orc_f32_to_f16(float(v)) for v in vals], np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(mine, vals.astype(np.float16).view(np.uint16))
    back = np.array([oracle.lib().orc_f16_to_f32(int(h)) for h in mine], np.float32)
    assert np.array_equal(back, mine.view(np.float16).astype(np.float32))


def test_quantize_is_byte_equal_to_gguf(oracle):
    z = np.load(GOLDEN / "q8_quant.npz")
    assert np.array_equal(oracle.q8_quantize(z["w"]), z["q8"])


def test_dequantize_is_exact(oracle):
    z = np.load(GOLDEN / "q8_quant.npz")
    w = oracle.q8_dequantize(z["q8"], *z["w"].shape)
    blocks = z["q8"].reshape(-1, 34)
    d = blocks[:, :2].copy().view(np.float16).astype(np.float32)
    q = blocks[:, 2:].copy().view(np.int8).astype(np.float32)
    assert np.array_equal(w.reshape(-1, 32), d * q)


@pytest.mark.parametrize("name", sorted(_gemm_cases()))
def test_gemm_is_bit_equal_to_the_reference_float_kernel(oracle, name):
    c = _gemm_cases()[name]
    m, n, k, n_off, cnt, gelu, has_res = (int(v) for v in c["meta"])
    res = c["res"] if has_res else None
    y = oracle.gemm_q8(c["x"], c["q8"], c["bias"], n, k, n_off, cnt, res,
                       oracle.ACT_GELU_ERF if gelu else oracle.ACT_NONE)
    if gelu:
        # finish_tile uses the AVX exp256 for full 16-column tiles and std::exp on the ragged edge.
        np.testing.assert_allclose(y, c["y"], rtol=0, atol=2e-6)
    else:
        assert np.array_equal(y, c["y"])


def test_panel_blob_matches_the_reference_dequantizer(oracle):
    if not oracle.have_ref():
        pytest.skip("reference library not built here")
    z = np.load(GOLDEN / "q8_quant.npz")
    w, q = z["w"], z["q8"]
    lin = oracle.RefLinear(q, None, w.shape[0], w.shape[1])
    assert np.array_equal(lin.dequantize(), oracle.q8_dequantize(q, w.shape[0], w.shape[1]))


def test_panel_conversion_rejects_inexact_minimum(oracle):
    # d = 600 makes -128 d overflow fp16, which tools/gguf_to_decoder.py:36-38 rejects.
    w = np.zeros((1, 32), np.float32)
    w[0, 0] = 127.0 * 600.0
    with pytest.raises(ValueError):
        oracle.q8_to_panels(oracle.q8_quantize(w), 1, 32)


def test_norms_and_activations_match_the_reference(oracle):
    z = np.load(GOLDEN / "ops.npz")
    rows, dim, heads, hd, lq, lk = (int(v) for v in z["meta"])
    np.testing.assert_allclose(oracle.norm_rows(z["x"], 1e-6), z["ln_plain"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(oracle.norm_rows(z["x"], 1e-6, z["gamma"], z["beta"]), z["ln_affine"], rtol=0,
                               atol=1e-6)
    np.testing.assert_allclose(oracle.norm_rows(z["x"], 1e-5, shift=z["shift"], scale=z["scale"]), z["ln_ada"],
                               rtol=0, atol=1e-6)
    got = oracle.rms_heads(z["qk"], heads, hd, z["qk_gamma"], col0=0)
    np.testing.assert_allclose(got[:, :dim], z["rms"][:, :dim], rtol=0, atol=2e-6)
    np.testing.assert_allclose(oracle.activate(z["gelu_in"], oracle.ACT_GELU_TANH), z["gelu_out"], rtol=0, atol=2e-6)


def test_attention_matches_the_reference(oracle):
    z = np.load(GOLDEN / "ops.npz")
    rows, dim, heads, hd, lq, lk = (int(v) for v in z["meta"])
    kv = z["att_kv"]
    out = oracle.attention(z["att_q"], np.ascontiguousarray(kv[:, :dim]), np.ascontiguousarray(kv[:, dim:]), heads, hd)
    np.testing.assert_allclose(out, z["att_out"], rtol=0, atol=2e-6)


def test_oracle_equals_live_reference_on_fresh_inputs(oracle):
    if not oracle.have_ref():
        pytest.skip("reference library not built here")
    rng = np.random.default_rng(99)
    for m, n, k in [(13, 50, 96), (64, 160, 512)]:
        w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
        q = oracle.q8_quantize(w)
        x = rng.normal(0, 1, (m, k)).astype(np.float32)
        b = rng.normal(0, 0.01, n).astype(np.float32)
        assert np.array_equal(oracle.gemm_q8(x, q, b, n, k), oracle.RefLinear(q, b, n, k).gemm(x))


def test_gaussian_heads(oracle):
    rng = np.random.default_rng(3)
    raw = rng.normal(0, 1, (50, 14)).astype(np.float32)
    raw[0, 6:10] = 0.0
    out = oracle.gaussian_heads(raw)
    np.testing.assert_array_equal(out[:, :3], raw[:, :3])
    np.testing.assert_allclose(out[:, 3:6], np.exp(raw[:, 3:6]), rtol=1e-6)
    r = raw[:, 6:10] * np.float32(0.1) + np.array([1, 0, 0, 0], np.float32)
    np.testing.assert_allclose(out[:, 6:10], r / np.linalg.norm(r, axis=1, keepdims=True), rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(out[0, 6:10], [1, 0, 0, 0])
    np.testing.assert_allclose(out[:, 10:], 1 / (1 + np.exp(-raw[:, 10:])), rtol=1e-6)


def test_reference_composed_block_matches_the_oracle_block(oracle):
    """The denoiser block composed of the reference's own compiled functions (the CPU baseline of the stack) against
    the oracle's restatement of the same composition."""
    if not oracle.have_ref():
        pytest.skip("oracle/_ref not built (no reference checkout)")
    rng = np.random.default_rng(21)
    D, heads, H, images, L = 256, 4, 1024, 2, 48
    layers = {}
    for name, (n, k) in {"qkv": (3 * D, D), "out": (D, D), "ff1": (H, D), "ff2": (D, H)}.items():
        layers[name] = (oracle.q8_quantize(rng.normal(0, 0.02, (n, k)).astype(np.float32)),
                        rng.normal(0, 0.01, n).astype(np.float32), n, k)
    layers["q_gamma"] = rng.normal(1, 0.1, D).astype(np.float32)
    layers["k_gamma"] = rng.normal(1, 0.1, D).astype(np.float32)
    x = rng.normal(0, 1, (images * L, D)).astype(np.float32)
    want = oracle.block_forward(x, layers, heads, images=images)
    got = oracle.RefBlock(layers, heads).forward_(x.copy(), images=images)
    rms = np.sqrt((want.astype(np.float64) ** 2).mean())
    assert np.abs(got - want).max() <= 1e-5 * rms


@pytest.mark.parametrize("m,n,k,n_off,cnt,gelu,res", [(5, 16, 32, 0, 16, 0, 0), (37, 48, 256, 0, 48, 0, 0),
                                                      (64, 256, 1024, 0, 256, 0, 0), (7, 100, 96, 0, 100, 0, 0),
                                                      (19, 96, 128, 16, 48, 1, 1), (3, 64, 64, 16, 40, 0, 1)])
def test_int8_activation_gemm_is_bit_equal_to_the_reference_vnni_kernel(oracle, m, n, k, n_off, cnt, gelu, res):
    """The restatement of the reference's second kernel (src/kernels.cpp:368-479, set_quant_kernel(1)) against the
    compiled reference itself: window (on the reference's 16-column panel boundaries, which its windows assume),
    residual and the erf GELU included."""
    if not oracle.have_ref():
        pytest.skip("oracle/_ref not built (no reference checkout)")
    rng = np.random.default_rng(m * n + k)
    q8 = oracle.q8_quantize(rng.normal(0, 0.02, (n, k)).astype(np.float32))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    x[0, :32] = 0.0  # an all-zero group: scale 0, codes 0
    b = rng.normal(0, 0.01, n).astype(np.float32)
    r = rng.normal(0, 1, (m, cnt)).astype(np.float32) if res else None
    mine = oracle.gemm_q8_int8act(x, q8, b, n, k, n_off, cnt, r, oracle.ACT_GELU_ERF if gelu else oracle.ACT_NONE)
    ref = oracle.RefLinear(q8, b, n, k).gemm(x, n_off, cnt, r, bool(gelu), mode=1)
    if gelu:
        np.testing.assert_allclose(mine, ref, rtol=0, atol=2e-6)  # the reference's exp256 vs std::exp, as above
    else:
        assert np.array_equal(mine, ref)
