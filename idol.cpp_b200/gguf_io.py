"""The Idol GGUF container on the host, for the packed linear layers, and the decoder cache's identity record.

* ``IdolGGUF``            - opens an Idol GGUF file with gguf-py as tools/idol_gguf.py:114-135 does: the
                            ``general.architecture`` must be ``idol`` with an embedded ``idol.config.json`` naming the
                            denoiser, decoder, decoder_gs and image_encoders configurations; every tensor is
                            ``idol.<component>.<name>`` for the four components, each present, no duplicates, only the
                            encodings the reference accepts.
* ``IdolGGUF.packed_linears(component)`` - every Q8_0, Q4_0 and Q4_K linear weight of a component as this package's
                            ``PackedLinear`` (the GGUF bytes kept packed; their ``fused`` path runs the sm_100a
                            kernels), with its bias expanded to a given dtype, as tools/idol_gguf.py:167-224
                            load_module_packed builds the reference's - without the upstream torch modules, which this
                            build does not have.
* ``check_decoder_cache`` - the identity record a decoder cache directory carries (tools/idol_generate.py:49-70):
                            version 1 and the SHA-256 digests of the model file, manifest.txt and weights.bin; a
                            cache whose record is missing or does not match raises ValueError, as the reference's does.

gguf-py is imported on first use, so the rest of the package does not need it.
"""
from __future__ import annotations

import hashlib
import json
import re
from collections import Counter
from pathlib import Path
from typing import Dict

import numpy as np
import torch

from .q8 import _GGML_Q4_0, _GGML_Q4_K, _GGML_Q8_0, PackedLinear

COMPONENTS = ("denoiser", "octree", "gaussian", "background")
PACKED_KINDS = (_GGML_Q8_0, _GGML_Q4_0, _GGML_Q4_K)


def _gguf():
    import gguf
    return gguf


def _supported(gguf):
    t = gguf.GGMLQuantizationType
    return {t.F32, t.F16, t.Q8_0, t.Q4_0, t.Q2_K, t.Q4_K, t.Q6_K, t.I8, t.I16, t.I32, t.I64}


_TENSOR_NAME = re.compile(r"idol\.([^.]+)\.(.+)")
_CONFIG_KEYS = ("denoiser", "decoder", "decoder_gs", "image_encoders")


def _text_field(reader, key):
    field = reader.get_field(key)
    return None if field is None else field.contents()


def _container_config(reader) -> dict:
    """Header rule: the architecture is `idol` and an embedded `idol.config.json` carries the configurations of the
    denoiser, both decoders and the image encoders."""
    text = _text_field(reader, "idol.config.json")
    if _text_field(reader, "general.architecture") != "idol" or text is None:
        raise ValueError("not an Idol GGUF file with an embedded configuration")
    config = json.loads(text)
    if set(_CONFIG_KEYS) - set(config):
        raise ValueError("incomplete Idol configuration")
    return config


def _components(tensors, encodings) -> Dict[str, Dict]:
    """Tensor rules: every name is `idol.<component>.<layer name>` with one of the four components; no name twice;
    only the encodings the reference's loader accepts; each component has at least one tensor. Returns
    component -> {layer name: tensor}."""
    keyed = [(_TENSOR_NAME.fullmatch(t.name), t) for t in tensors]
    stray = next((t.name for m, t in keyed if m is None or m.group(1) not in COMPONENTS), None)
    if stray is not None:
        raise ValueError("unexpected tensor in Idol GGUF: " + stray)
    counts = Counter(t.name for _, t in keyed)
    bad = next((t.name for _, t in keyed if counts[t.name] > 1 or t.tensor_type not in encodings), None)
    if bad is not None:
        raise ValueError("duplicate tensor or unsupported GGUF encoding: " + bad)
    table = {c: {m.group(2): t for m, t in keyed if m.group(1) == c} for c in COMPONENTS}
    if not all(table.values()):
        raise ValueError("Idol GGUF is missing a component")
    return table


class IdolGGUF:
    """An Idol GGUF file opened with gguf-py and checked against the container rules of tools/idol_gguf.py:114-135
    (same error messages): `config` is the embedded configuration, `tensors[component][layer name]` the tensors."""

    def __init__(self, path):
        gguf = _gguf()
        self.path = Path(path)
        self.reader = gguf.GGUFReader(self.path)
        self.config = _container_config(self.reader)
        self.tensors: Dict[str, Dict] = _components(self.reader.tensors, _supported(gguf))

    def packed_linears(self, component: str, bias_dtype=torch.float32) -> Dict[str, PackedLinear]:
        """layer name -> PackedLinear for every 2-D Q8_0 / Q4_0 / Q4_K `<layer>.weight` of the component; a scale
        that is not finite raises ValueError (tools/idol_gguf.py:20-38 validate_tensor_values). The bias is
        expanded to `bias_dtype`: fused calls want it in the activation dtype, as the reference's modules hold it."""
        gguf = _gguf()
        if component not in self.tensors:
            raise ValueError("unknown component: " + component)
        source = self.tensors[component]
        out = {}
        for name, tensor in source.items():
            if int(tensor.tensor_type) not in PACKED_KINDS:
                continue
            if not name.endswith(".weight") or len(tensor.shape) != 2:
                raise ValueError("quantized tensor is not a linear weight: " + name)
            block = {_GGML_Q8_0: 34, _GGML_Q4_0: 18, _GGML_Q4_K: 144}[int(tensor.tensor_type)]
            scale_offsets = (0, 2) if int(tensor.tensor_type) == _GGML_Q4_K else (0,)
            raw = np.asarray(tensor.data).reshape(-1, block)
            for off in scale_offsets:
                if not np.isfinite(np.ascontiguousarray(raw[:, off:off + 2]).view("<f2")).all():
                    raise ValueError(f"non-finite value in {component}.{name}")
            layer = name[:-len(".weight")]
            bias = None
            if layer + ".bias" in source:
                b = source[layer + ".bias"]
                values = gguf.dequantize(b.data, b.tensor_type)
                bias = torch.from_numpy(np.array(values, dtype=np.float32, copy=True)).reshape(-1).to(bias_dtype)
            out[layer] = PackedLinear(tensor, bias)
        return out


def _digest(path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as stream:
        for chunk in iter(lambda: stream.read(4 * 1024 * 1024), b""):
            h.update(chunk)
    return h.hexdigest()


def cache_identity(model_path, export_dir) -> Dict:
    """The identity record of a decoder cache directory holding the export made from `model_path`."""
    export_dir = Path(export_dir)
    return {"version": 1, "model_sha256": _digest(model_path),
            "manifest_sha256": _digest(export_dir / "manifest.txt"),
            "weights_sha256": _digest(export_dir / "weights.bin")}


def check_decoder_cache(model_path, export_dir) -> Path:
    """Returns export_dir if its idol-cache.json matches the model file and the export's bytes; raises ValueError
    otherwise (a directory without a completed record, or a record for other bytes)."""
    export_dir = Path(export_dir)
    record = export_dir / "idol-cache.json"
    if not record.is_file():
        raise ValueError("decoder cache exists without a completed identity record")
    if json.loads(record.read_text(encoding="utf-8")) != cache_identity(model_path, export_dir):
        raise ValueError("decoder cache does not match this model or its recorded bytes")
    return export_dir


def write_decoder_cache_identity(model_path, export_dir) -> Path:
    """Completes a freshly written export directory with its identity record (created exclusively, as the reference
    does, so a second writer fails instead of overwriting)."""
    export_dir = Path(export_dir)
    with (export_dir / "idol-cache.json").open("x", encoding="utf-8") as stream:
        json.dump(cache_identity(model_path, export_dir), stream, indent=2)
    return export_dir
