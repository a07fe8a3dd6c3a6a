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


class IdolGGUF:
    def __init__(self, path):
        gguf = _gguf()
        self.path = Path(path)
        self.reader = gguf.GGUFReader(self.path)
        arch = self.reader.get_field("general.architecture")
        config = self.reader.get_field("idol.config.json")
        if arch is None or arch.contents() != "idol" or config is None:
            raise ValueError("not an Idol GGUF file with an embedded configuration")
        self.config = json.loads(config.contents())
        if not all(k in self.config for k in ("denoiser", "decoder", "decoder_gs", "image_encoders")):
            raise ValueError("incomplete Idol configuration")
        supported = _supported(gguf)
        self.tensors: Dict[str, Dict] = {name: {} for name in COMPONENTS}
        for tensor in self.reader.tensors:
            parts = tensor.name.split(".", 2)
            if len(parts) != 3 or parts[0] != "idol" or parts[1] not in self.tensors or not parts[2]:
                raise ValueError("unexpected tensor in Idol GGUF: " + tensor.name)
            group = self.tensors[parts[1]]
            if parts[2] in group or tensor.tensor_type not in supported:
                raise ValueError("duplicate tensor or unsupported GGUF encoding: " + tensor.name)
            group[parts[2]] = tensor
        if any(not values for values in self.tensors.values()):
            raise ValueError("Idol GGUF is missing a component")

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
