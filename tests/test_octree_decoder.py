"""The octree decoder (next-row (f)3): Decoders::octree_logits and sample_anchors (src/decoders.cpp:242-282,
335-391), and Decoders::decode (:435-445) over both decoders.

CPU: the oracle's octree_logits composition equals the reference's own (compiled from its sources, float kernel) on a
random-weight native export within 1e-5 x rms; the library's host sampler, driven level by level with the reference's
own logits, reproduces the reference's sample_anchors bit for bit (same generator, draw order and arithmetic).
GPU: OctreeDecoder.from_native_export: logits within 2e-2 x rms of the oracle at several resolutions; sample_anchors
equal to the host sampler driven with those GPU logits, and at one level within 1% of the points of the sampler driven
with the oracle's logits; decode end to end.
"""
import numpy as np
import pytest
import torch

from native_export import write_decoders_export


def _cond(rows, seed):
    return np.random.default_rng(seed).normal(0, 1, (rows, 16)).astype(np.float32)


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).have_ref()")
def test_oracle_octree_logits_matches_the_reference(oracle, tmp_path):
    _, octd = write_decoders_export(tmp_path, oracle, D=96, heads=2, gs_blocks=0, cond=16, per_anchor=4, seed=1,
                                    oct_blocks=2, with_octree=True)
    ref = oracle.RefDecoders(tmp_path)
    x = np.random.default_rng(0).uniform(0, 1, (40, 3)).astype(np.float32)
    cond = _cond(70, 1)
    for res in (2.0, 16.0, 256.0):
        want = ref.octree_logits(x, res, cond)
        got = oracle.octree_logits(x, res, cond, octd, 2)
        rms = np.sqrt((want.astype(np.float64) ** 2).mean())
        assert np.abs(got - want).max() <= 1e-5 * rms, res


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).have_ref()")
@pytest.mark.parametrize("num_points,level,seed", [(1, 1, 0), (500, 3, 7), (2000, 5, 123456789)])
def test_host_sampler_reproduces_the_reference_sample_anchors(pkg, oracle, tmp_path, num_points, level, seed):
    from idol_b200.native import OctreeSampler
    write_decoders_export(tmp_path, oracle, D=96, heads=2, gs_blocks=0, cond=16, per_anchor=4, seed=2, oct_blocks=1)
    ref = oracle.RefDecoders(tmp_path)
    cond = _cond(50, 3)
    want = ref.sample_anchors(cond, num_points, level, seed)
    got = OctreeSampler(num_points, level, seed).run(lambda centres, res: ref.octree_logits(centres, res, cond))
    assert np.array_equal(got, want)


def test_host_sampler_argument_errors(pkg):
    from idol_b200.native import OctreeSampler
    for bad in ((0, 3), (10, 0), (10, 21)):
        with pytest.raises(Exception):
            OctreeSampler(bad[0], bad[1], 0)


def _leaf_cells(points, level):
    return np.floor(points.astype(np.float64) * (1 << level)).astype(np.int64)


@pytest.mark.gpu
def test_octree_decoder_from_the_native_export(pkg, oracle, cuda, tmp_path):
    from idol_b200.native import OctreeDecoder, OctreeSampler
    _, octd = write_decoders_export(tmp_path, oracle, D=256, heads=4, gs_blocks=0, cond=16, per_anchor=32, seed=5,
                                    oct_blocks=2, with_octree=True)
    dec = OctreeDecoder.from_native_export(tmp_path, cuda)
    cond = _cond(300, 4)
    x = np.random.default_rng(6).uniform(0, 1, (200, 3)).astype(np.float32)
    for res in (2.0, 32.0, 1024.0):
        got = dec.logits(torch.from_numpy(x), res, torch.from_numpy(cond)).cpu().numpy()
        want = oracle.octree_logits(x, res, cond, octd, 4)
        rms = np.sqrt((want.astype(np.float64) ** 2).mean())
        err = np.abs(got - want).max()
        assert np.isfinite(got).all() and err <= 2e-2 * rms, f"resolution {res}: {err:.3e} > 2e-2 x {rms:.3e}"
    # sample_anchors is the host sampler (pinned to the reference above) driven by these logits: the library's loop
    # equals the sampler driven from Python with the same GPU logits, bit for bit.
    num_points, level, seed = 3000, 5, 11
    pts = dec.sample_anchors(torch.from_numpy(cond), num_points, level, seed)
    assert pts.shape == (num_points, 3) and np.isfinite(pts).all() and (pts >= 0).all() and (pts <= 1).all()
    cond_t = torch.from_numpy(cond).to(cuda)
    driven = OctreeSampler(num_points, level, seed).run(
        lambda c, r: dec.logits(torch.from_numpy(c), r, cond_t).cpu().numpy())
    assert np.array_equal(pts, driven)
    # One level against the oracle's logits: bf16 logits move at most a few of the root's points between children
    # (deeper levels diverge by design: a cell that changes shifts every later cell's draw).
    one = _leaf_cells(dec.sample_anchors(cond_t, num_points, 1, seed), 1)
    ref = _leaf_cells(OctreeSampler(num_points, 1, seed).run(lambda c, r: oracle.octree_logits(c, r, cond, octd, 4)), 1)
    ca = np.bincount(one @ np.array([1, 2, 4]), minlength=8)
    cb = np.bincount(ref @ np.array([1, 2, 4]), minlength=8)
    assert np.abs(ca - cb).sum() / 2 <= 0.01 * num_points, (ca, cb)


@pytest.mark.gpu
def test_decode_end_to_end(pkg, oracle, cuda, tmp_path):
    from idol_b200.native import GaussianDecoder, OctreeDecoder, decode
    write_decoders_export(tmp_path, oracle, D=256, heads=4, gs_blocks=1, cond=16, per_anchor=32, seed=8,
                          oct_blocks=1)
    octree = OctreeDecoder.from_native_export(tmp_path, cuda)
    gaussian = GaussianDecoder.from_native_export(tmp_path, cuda)
    cloud = decode(octree, gaussian, torch.from_numpy(_cond(200, 9)), 32 * 100 + 5, 4, 3)
    torch.cuda.synchronize()
    n = 100 * 32
    assert {k: tuple(v.shape) for k, v in cloud.items()} == {"xyz": (n, 3), "f_dc": (n, 3), "scale": (n, 3),
                                                            "rotation": (n, 4), "opacity": (n,)}
    for k, v in cloud.items():
        assert torch.isfinite(v).all(), k
    assert torch.allclose(cloud["rotation"].norm(dim=1), torch.ones(n, device=cuda), atol=1e-5)
    assert ((cloud["opacity"] > 0) & (cloud["opacity"] < 1)).all()
