"""The Gaussian decoder (next-row (f)1): Decoders::gaussian_features and to_gaussians (src/decoders.cpp:284-316,
393-433) over the native export (src/weights.cpp:25-104).

CPU: the oracle's composition (pos_embed, in_proj, the blocks with their cross-attention, LN, out_proj) equals the
reference's own Decoders::gaussian_features, compiled from its sources, on a random-weight export that
tests/native_export.py writes (float kernel, as production forces: within 1e-5 x rms); its to_gaussians within one
fp32 ulp; the export reader and the panel -> Q8_0 conversion are exact.
GPU: GaussianDecoder.from_native_export runs the same export on sm_100a; features within 2e-2 x rms of the oracle
(bf16 activations), Gaussian parameters within 1e-2 relative (north_star) with the group RMS as the floor.
"""
import numpy as np
import pytest
import torch

from native_export import write_decoders_export


def _inputs(rows, cond_rows, cond_dim, seed):
    rng = np.random.default_rng(seed)
    return (rng.uniform(0, 1, (rows, 3)).astype(np.float32),
            rng.normal(0, 1, (cond_rows, cond_dim)).astype(np.float32))


def test_native_export_reader_and_panel_conversion(pkg, oracle, tmp_path):
    from idol_b200.native import panels_to_q8, read_native_export
    dec = write_decoders_export(tmp_path, oracle, D=96, heads=2, gs_blocks=1, cond=16, per_anchor=4, seed=3)
    ex = read_native_export(tmp_path)
    assert ex["config"] == {"dim": 96, "heads": 2, "oct_blocks": 0, "gs_blocks": 1, "cond": 16, "per_anchor": 4}
    assert np.array_equal(ex["tensors"]["gs.in_proj.weight"], dec["in_w"])
    o, i, bits, group, blob = ex["qtensors"]["gs.out_proj.weight"]
    assert (o, i, bits, group) == (60, 96, 8, 32)
    assert np.array_equal(panels_to_q8(blob, o, i), dec["out"][0].reshape(-1))
    rng = np.random.default_rng(0)
    for out, inp in ((1, 32), (17, 64), (33, 96)):
        q8 = oracle.q8_quantize(rng.normal(0, 0.1, (out, inp)).astype(np.float32))
        assert np.array_equal(panels_to_q8(oracle.q8_to_panels(q8, out, inp), out, inp), q8.reshape(-1))


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).have_ref()")
@pytest.mark.parametrize("blocks", [0, 2])
def test_oracle_composition_matches_the_reference_decoders(oracle, tmp_path, blocks):
    dec = write_decoders_export(tmp_path, oracle, D=96, heads=2, gs_blocks=blocks, cond=16, per_anchor=4, seed=1)
    ref = oracle.RefDecoders(tmp_path)
    pts, cond = _inputs(50, 70, 16, 0)
    want = ref.gaussian_features(pts, cond, 60, mode=0)
    got = oracle.gaussian_features(pts, cond, dec, 2)
    rms = np.sqrt((want.astype(np.float64) ** 2).mean())
    assert np.abs(got - want).max() <= 1e-5 * rms
    g_ref = ref.to_gaussians(pts, want, 4)
    g = oracle.to_gaussians(pts, want, 4, dec["perturbation"], dec["base_offset_scale"])
    for k in g:
        np.testing.assert_allclose(g[k], g_ref[k], rtol=2.5e-7, atol=2.5e-7, err_msg=k)


@pytest.mark.gpu
def test_gaussian_decoder_from_the_native_export(pkg, oracle, cuda, tmp_path):
    from idol_b200.native import GaussianDecoder
    D, heads, G = 256, 4, 32
    dec = write_decoders_export(tmp_path, oracle, D=D, heads=heads, gs_blocks=2, cond=16, per_anchor=G, seed=7)
    gd = GaussianDecoder.from_native_export(tmp_path, cuda)
    pts, cond = _inputs(300, 500, 16, 1)
    feats = gd.features(torch.from_numpy(pts), torch.from_numpy(cond))
    torch.cuda.synchronize()
    want = oracle.gaussian_features(pts, cond, dec, heads)
    got = feats.cpu().numpy()
    rms = np.sqrt((want.astype(np.float64) ** 2).mean())
    err = np.abs(got - want).max()
    assert np.isfinite(got).all() and err <= 2e-2 * rms, f"features: {err:.3e} > 2e-2 x {rms:.3e}"
    # to_gaussians on the oracle's features isolates the activation kernel from the features' bf16 error.
    g = {k: v.cpu().numpy() for k, v in gd.to_gaussians(torch.from_numpy(pts), torch.from_numpy(want)).items()}
    g_ref = oracle.to_gaussians(pts, want, G, dec["perturbation"], dec["base_offset_scale"])
    for k in g_ref:
        floor = np.sqrt((g_ref[k].astype(np.float64) ** 2).mean())
        rel = (np.abs(g[k] - g_ref[k]) / np.maximum(np.abs(g_ref[k]), floor)).max()
        assert rel <= 1e-2, f"{k}: relative error {rel:.2e}"
    # End to end: the GPU's own features through the GPU's activation, against the oracle's whole chain.
    g_gpu = {k: v.cpu().numpy() for k, v in gd.to_gaussians(torch.from_numpy(pts), feats).items()}
    for k in ("xyz", "rotation", "opacity"):
        floor = np.sqrt((g_ref[k].astype(np.float64) ** 2).mean())
        rel = (np.abs(g_gpu[k] - g_ref[k]) / np.maximum(np.abs(g_ref[k]), floor)).max()
        assert rel <= 5e-2, f"{k} end to end: relative error {rel:.2e}"
