"""Host-side logic that needs no GPU: the octree sampler on synthetic logits, and the native export reader's
refusals of malformed files."""
import numpy as np
import pytest


def _run(sampler_cls, n, level, seed, logits_fn):
    s = sampler_cls(n, level, seed)
    return s.run(logits_fn)


def test_sampler_properties(pkg):
    from idol_b200.native import OctreeSampler
    rng = np.random.default_rng(0)
    table = {}

    def logits(centres, res):
        # deterministic per (cell, resolution), so two runs see the same logits
        out = np.empty((centres.shape[0], 8), np.float32)
        for i, c in enumerate(centres):
            key = (tuple(np.round(c * res).astype(int)), res)
            if key not in table:
                table[key] = rng.normal(0, 2, 8).astype(np.float32)
            out[i] = table[key]
        return out

    n, level = 777, 4
    a = _run(OctreeSampler, n, level, 5, logits)
    b = _run(OctreeSampler, n, level, 5, logits)
    c = _run(OctreeSampler, n, level, 6, logits)
    assert a.shape == (n, 3) and np.array_equal(a, b) and not np.array_equal(a, c)
    assert (a >= 0).all() and (a < 1).all()
    # points of one leaf cell are contiguous and inside it
    cells = np.floor(a * (1 << level)).astype(np.int64)
    seen, last = set(), None
    for cell in map(tuple, cells):
        if cell != last:
            assert cell not in seen, "a leaf cell's points are not contiguous"
            seen.add(cell)
            last = cell


def test_sampler_follows_a_certain_child(pkg):
    """Logits that put all mass on child 5 (x odd, y even, z odd) at every level send every point to one leaf."""
    from idol_b200.native import OctreeSampler
    level = 3

    def logits(centres, res):
        out = np.full((centres.shape[0], 8), -60.0, np.float32)
        out[:, 5] = 60.0
        return out

    pts = _run(OctreeSampler, 100, level, 1, logits)
    cells = np.unique(np.floor(pts * (1 << level)).astype(np.int64), axis=0)
    assert cells.tolist() == [[7, 0, 7]]


def test_sampler_level_protocol(pkg):
    from idol_b200.native import OctreeSampler
    s = OctreeSampler(10, 2, 0)
    n, res = s.cells()
    assert (n, res) == (1, 2.0)
    assert np.allclose(s.centres(), [[0.5, 0.5, 0.5]])
    with pytest.raises(Exception):
        s.points()  # levels remain
    s.step(np.zeros((1, 8), np.float32))
    n, res = s.cells()
    assert res == 4.0 and 1 <= n <= 8
    s.step(np.zeros((n, 8), np.float32))
    assert s.cells()[0] == 0
    with pytest.raises(Exception):
        s.step(np.zeros((1, 8), np.float32))  # every level done
    assert s.points().shape == (10, 3)


def _write(path, manifest, blob=b"\0" * 64):
    path.mkdir(parents=True, exist_ok=True)
    (path / "manifest.txt").write_text(manifest)
    (path / "weights.bin").write_bytes(blob)


def test_native_export_reader_refusals(pkg, tmp_path):
    from idol_b200.native import panels_to_q8, read_native_export
    _write(tmp_path / "a", "")
    with pytest.raises(ValueError, match="empty"):
        read_native_export(tmp_path / "a")
    _write(tmp_path / "b", "octree 1 2 3\n")
    with pytest.raises(ValueError, match="first line"):
        read_native_export(tmp_path / "b")
    _write(tmp_path / "c", "decoders 96 2 0 0 16 4\nw 1 4 0 12\n")
    with pytest.raises(ValueError, match="byte count"):
        read_native_export(tmp_path / "c")
    _write(tmp_path / "d", "decoders 96 2 0 0 16 4\nw 1 4 60 16\n")
    with pytest.raises(ValueError, match="outside"):
        read_native_export(tmp_path / "d")
    _write(tmp_path / "e", "decoders 96 2 0 0 16 4\nqtensor q 16 32 8 32 0 1000\n")
    with pytest.raises(ValueError, match="outside"):
        read_native_export(tmp_path / "e")
    _write(tmp_path / "f", "decoders 96 2 0 0 16 4\nrep 1 2 3 4 5 6 7 8 9\ncase 8 16 3\nw 1 4 0 16\n")
    ex = read_native_export(tmp_path / "f")
    assert ex["rep"] == tuple(float(v) for v in range(1, 10)) and ex["case"] == (8, 16, 3)
    assert ex["tensors"]["w"].shape == (4,)
    # a panel blob whose minimums are not -128 x scale is not a Q8_0 matrix
    blob = np.zeros(576, np.uint8)
    blob[0:2] = np.array([1.0], np.float16).view(np.uint8)
    blob[32:34] = np.array([-100.0], np.float16).view(np.uint8)
    with pytest.raises(ValueError, match="-128"):
        panels_to_q8(blob, 16, 32)
    with pytest.raises(ValueError, match="size"):
        panels_to_q8(blob[:500], 16, 32)
