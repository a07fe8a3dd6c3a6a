"""The Idol GGUF container and the decoder cache's identity record (idol.cpp_b200/gguf_io.py), on the CPU.

A small Idol GGUF is written with gguf-py's own writer: the container checks of tools/idol_gguf.py:114-135 hold
(architecture, embedded configuration, the four components, tensor naming, encodings), the packed linears come back as
PackedLinear layers whose expansion equals gguf-py's dequantize exactly, a non-finite scale is refused, and the cache
record of tools/idol_generate.py:49-70 accepts its own export and refuses changed bytes or a missing record.
"""
import json

import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")


def _write(path, tensors, arch="idol", config=True):
    w = gguf.GGUFWriter(str(path), arch)
    if config:
        w.add_string("idol.config.json", json.dumps({"denoiser": {}, "decoder": {}, "decoder_gs": {},
                                                     "image_encoders": {}}))
    for name, (data, kind) in tensors.items():
        if kind is None:
            w.add_tensor(name, data)
        else:
            w.add_tensor(name, data, raw_shape=data.shape, raw_dtype=kind)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def _model(rng):
    Q8, Q4 = gguf.GGMLQuantizationType.Q8_0, gguf.GGMLQuantizationType.Q4_0
    w1 = rng.normal(0, 0.02, (64, 96)).astype(np.float32)
    w2 = rng.normal(0, 0.02, (32, 128)).astype(np.float32)
    t = {"idol.gaussian.blocks.0.mlp.mlp.0.weight": (gguf.quantize(w1, Q8), Q8),
         "idol.gaussian.blocks.0.mlp.mlp.0.bias": (rng.normal(0, 0.01, 64).astype(np.float32), None),
         "idol.gaussian.out_proj.weight": (gguf.quantize(w2, Q4), Q4),
         "idol.gaussian.norm.weight": (np.ones(96, np.float32), None)}
    for c in ("denoiser", "octree", "background"):
        t[f"idol.{c}.scale"] = (np.ones(4, np.float32), None)
    return t


def test_packed_linears_expand_exactly(pkg, tmp_path):
    from idol_b200.gguf_io import IdolGGUF
    tensors = _model(np.random.default_rng(0))
    _write(tmp_path / "m.gguf", tensors)
    g = IdolGGUF(tmp_path / "m.gguf")
    layers = g.packed_linears("gaussian", bias_dtype=torch.bfloat16)
    assert set(layers) == {"blocks.0.mlp.mlp.0", "out_proj"}
    a = layers["blocks.0.mlp.mlp.0"]
    assert a.shape == (64, 96) and a.bias.dtype == torch.bfloat16
    data, kind = tensors["idol.gaussian.blocks.0.mlp.mlp.0.weight"]
    assert np.array_equal(a.dequantize(torch.float32).numpy(), gguf.dequantize(data, kind).reshape(64, 96))
    b = layers["out_proj"]
    assert b.bias is None
    data, kind = tensors["idol.gaussian.out_proj.weight"]
    assert np.array_equal(b.dequantize(torch.float32).numpy(), gguf.dequantize(data, kind).reshape(32, 128))


def test_container_checks(pkg, tmp_path):
    from idol_b200.gguf_io import IdolGGUF
    rng = np.random.default_rng(1)
    t = _model(rng)
    _write(tmp_path / "a.gguf", t, arch="llama")
    with pytest.raises(ValueError, match="not an Idol GGUF"):
        IdolGGUF(tmp_path / "a.gguf")
    _write(tmp_path / "b.gguf", t, config=False)
    with pytest.raises(ValueError, match="not an Idol GGUF"):
        IdolGGUF(tmp_path / "b.gguf")
    t2 = dict(t)
    del t2["idol.background.scale"]
    _write(tmp_path / "c.gguf", t2)
    with pytest.raises(ValueError, match="missing a component"):
        IdolGGUF(tmp_path / "c.gguf")
    t3 = dict(t)
    t3["idol.unknown.x"] = (np.ones(2, np.float32), None)
    _write(tmp_path / "d.gguf", t3)
    with pytest.raises(ValueError, match="unexpected tensor"):
        IdolGGUF(tmp_path / "d.gguf")
    t4 = dict(t)
    data, kind = t4["idol.gaussian.blocks.0.mlp.mlp.0.weight"]
    bad = data.copy()
    bad[0, 0:2] = np.array([np.inf], np.float16).view(np.uint8)
    t4["idol.gaussian.blocks.0.mlp.mlp.0.weight"] = (bad, kind)
    _write(tmp_path / "e.gguf", t4)
    with pytest.raises(ValueError, match="non-finite"):
        IdolGGUF(tmp_path / "e.gguf").packed_linears("gaussian")


def test_decoder_cache_identity(pkg, tmp_path):
    from idol_b200.gguf_io import check_decoder_cache, write_decoder_cache_identity
    model = tmp_path / "model.gguf"
    model.write_bytes(b"model bytes")
    cache = tmp_path / "cache"
    cache.mkdir()
    (cache / "manifest.txt").write_text("decoders 256 4 0 0 16 32\n")
    (cache / "weights.bin").write_bytes(b"\0" * 64)
    with pytest.raises(ValueError, match="without a completed identity record"):
        check_decoder_cache(model, cache)
    write_decoder_cache_identity(model, cache)
    assert check_decoder_cache(model, cache) == cache
    with pytest.raises(FileExistsError):
        write_decoder_cache_identity(model, cache)
    (cache / "weights.bin").write_bytes(b"\1" * 64)
    with pytest.raises(ValueError, match="does not match"):
        check_decoder_cache(model, cache)


def test_container_checks_configuration_and_encodings(pkg, tmp_path):
    from idol_b200.gguf_io import IdolGGUF
    t = _model(np.random.default_rng(2))
    w = gguf.GGUFWriter(str(tmp_path / "f.gguf"), "idol")
    w.add_string("idol.config.json", json.dumps({"denoiser": {}, "decoder": {}}))
    for name, (data, kind) in t.items():
        w.add_tensor(name, data) if kind is None else w.add_tensor(name, data, raw_shape=data.shape, raw_dtype=kind)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ValueError, match="incomplete Idol configuration"):
        IdolGGUF(tmp_path / "f.gguf")
    t2 = dict(t)
    t2["idol.octree.odd"] = (np.zeros(44, np.uint8), gguf.GGMLQuantizationType.Q5_0)  # an encoding the loader refuses
    _write(tmp_path / "g.gguf", t2)
    with pytest.raises(ValueError, match="unsupported GGUF encoding: idol.octree.odd"):
        IdolGGUF(tmp_path / "g.gguf")
