"""Writes random-weight native exports of the reference's decoders (manifest.txt + weights.bin, the format
src/weights.cpp:25-104 reads and tools/export_idol.py writes) and returns the same weights in the oracle's and the GPU
compositions' terms. Test infrastructure: the export is how the reference's own Decoders::gaussian_features and
to_gaussians are run on the weights the GPU path runs on.

Quantized matrices go in as `qtensor` lines holding the idol panel blob (8 bits, group 32) converted from Q8_0 blocks
(tools/gguf_to_decoder.py), so the reference and the GPU path multiply by the same Q8_0 weights; `to_kv` (depth =
the condition width) and the 3-deep `in_proj` stay dense fp32 tensors, as in the real export.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np


def write_decoders_export(path, oracle, D=256, heads=4, gs_blocks=2, cond=16, per_anchor=32, seed=0, oct_blocks=0,
                          with_octree=False):
    """Returns the Gaussian decoder as a dict: in_w [D, 3], in_b, input/out (q8, bias, N, K), freqs, perturbation,
    base_offset_scale, blocks (list of layer dicts for oracle.gs_block_forward). With with_octree, returns
    (gaussian dict, octree dict) - the octree dict as oracle.octree_logits takes it."""
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    lines = [f"decoders {D} {heads} {oct_blocks} {gs_blocks} {cond} {per_anchor}",
             "rep 1.5 0.0009 0.004 0.1 1 1 1 1 0.1"]
    blob = bytearray()

    def put(data: bytes):
        off = len(blob)
        blob.extend(data)
        return off, len(data)

    def tensor(name, a):
        a = np.ascontiguousarray(a, dtype=np.float32)
        off, nb = put(a.tobytes())
        lines.append(f"{name} {a.ndim} {' '.join(str(d) for d in a.shape)} {off} {nb}")

    def dense(prefix, out, inp, scale):
        w = rng.normal(0, scale, (out, inp)).astype(np.float32)
        b = rng.normal(0, 0.01, out).astype(np.float32)
        tensor(prefix + ".weight", w)
        tensor(prefix + ".bias", b)
        return w, b

    def quant(prefix, out, inp, scale=0.02):
        q8 = oracle.q8_quantize(rng.normal(0, scale, (out, inp)).astype(np.float32))
        b = rng.normal(0, 0.01, out).astype(np.float32)
        off, nb = put(oracle.q8_to_panels(q8, out, inp).tobytes())
        lines.append(f"qtensor {prefix}.weight {out} {inp} 8 32 {off} {nb}")
        tensor(prefix + ".bias", b)
        return (q8, b, out, inp)

    def vec(name, n, mean=1.0, sd=0.1):
        v = rng.normal(mean, sd, n).astype(np.float32)
        tensor(name, v)
        return v

    fd = D // 3 // 2
    freqs = (2.0 ** np.linspace(0, 10, fd)).astype(np.float32)
    # The octree decoder (src/decoders.cpp:163-175, 200-202).
    octd = {"freqs": freqs}
    octd["in_w"], octd["in_b"] = dense("oct.in_proj", D, 3, 0.5)
    octd["input"] = quant("oct.input_layer", D, D, 0.05)
    octd["l1"] = quant("oct.l_embedder.mlp.0", D, 256, 0.1)
    octd["l2"] = quant("oct.l_embedder.mlp.2", D, D, 0.05)
    octd["ada"] = quant("oct.adaLN_modulation.1", 6 * D, D, 0.05)
    octd["out"] = quant("oct.out_proj", 8, D, 0.1)
    tensor("oct.pos_embedder.freqs", freqs)
    octd["level_freqs"] = np.exp(-np.log(1024.0) * np.arange(128) / 128).astype(np.float32)
    tensor("oct.l_embedder.freqs", octd["level_freqs"])
    octd["blocks"] = []
    for i in range(oct_blocks):
        p = f"oct.blocks.{i}."
        L = {"cq": quant(p + "cross_attn.to_q", D, D)}
        L["kv_w"], L["kv_b"] = dense(p + "cross_attn.to_kv", 2 * D, cond, 0.25)
        L["co"] = quant(p + "cross_attn.to_out", D, D)
        L["cq_gamma"] = vec(p + "cross_attn.q_rms_norm.gamma", D)
        L["ck_gamma"] = vec(p + "cross_attn.k_rms_norm.gamma", D)
        L["ff1"] = quant(p + "mlp.mlp.0", 4 * D, D)
        L["ff2"] = quant(p + "mlp.mlp.2", D, 4 * D)
        octd["blocks"].append(L)

    dec = {"freqs": freqs}
    dec["in_w"], dec["in_b"] = dense("gs.in_proj", D, 3, 0.5)
    dec["input"] = quant("gs.input_layer", D, D, 0.05)
    dec["out"] = quant("gs.out_proj", per_anchor * 15, D, 0.05)
    dec["perturbation"] = vec("gs.points_offset_perturbation", per_anchor * 3, 0.0, 0.1)
    dec["base_offset_scale"] = float(vec("gs.base_offset_scale", 1, -1.0, 0.1)[0])
    tensor("gs.pos_embedder.freqs", freqs)
    dec["blocks"] = []
    for i in range(gs_blocks):
        p = f"gs.blocks.{i}."
        L = {"qkv": quant(p + "self_attn.to_qkv", 3 * D, D), "out": quant(p + "self_attn.to_out", D, D),
             "q_gamma": vec(p + "self_attn.q_rms_norm.gamma", D), "k_gamma": vec(p + "self_attn.k_rms_norm.gamma", D),
             "cq": quant(p + "cross_attn.to_q", D, D)}
        L["kv_w"], L["kv_b"] = dense(p + "cross_attn.to_kv", 2 * D, cond, 0.25)
        L["co"] = quant(p + "cross_attn.to_out", D, D)
        L["cq_gamma"] = vec(p + "cross_attn.q_rms_norm.gamma", D)
        L["ck_gamma"] = vec(p + "cross_attn.k_rms_norm.gamma", D)
        L["norm2_gamma"] = vec(p + "norm2.weight", D)
        L["norm2_beta"] = vec(p + "norm2.bias", D, 0.0, 0.1)
        L["ff1"] = quant(p + "mlp.mlp.0", 4 * D, D)
        L["ff2"] = quant(p + "mlp.mlp.2", D, 4 * D)
        dec["blocks"].append(L)
    (path / "manifest.txt").write_text("\n".join(lines) + "\n")
    (path / "weights.bin").write_bytes(bytes(blob))
    return (dec, octd) if with_octree else dec
