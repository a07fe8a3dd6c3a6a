"""The reference's native decoder export (manifest.txt + weights.bin, src/weights.cpp:25-104) read on the host and
uploaded once, and the Gaussian decoder built from it on the GPU.

* ``read_native_export``   - parses manifest.txt (the ``decoders`` config line, ``rep``, ``case``, float32 tensors and
                             ``qtensor`` panel blobs) and reads weights.bin, as src/weights.cpp:25-104 does.
* ``panels_to_q8``         - an 8-bit, group-32 idol panel blob (tools/idolq.py:137-166) whose minimums are exactly
                             -128 x scale - the blobs tools/gguf_to_decoder.py:16-40 makes from GGUF Q8_0 - back into
                             the GGUF Q8_0 bytes it came from (bit-exact); other blobs raise ValueError.
* ``GaussianDecoder``      - Decoders::gaussian_features and Decoders::to_gaussians (src/decoders.cpp:284-316,
                             393-433) over resident weights (idol_b200_gs_decoder_*): Q8_0 matrices in the tiled layout,
                             the dense fp32 ``in_proj`` and ``to_kv`` as they are.
* ``OctreeDecoder``        - Decoders::octree_logits and sample_anchors (src/decoders.cpp:242-282, 335-391)
                             (idol_b200_oct_*): the logits on the GPU, the resampling on the host.
* ``OctreeSampler``        - the host half of sample_anchors alone (idol_b200_oct_sampler_*), for any logits source.
* ``decode``               - Decoders::decode (src/decoders.cpp:435-445): sample_anchors, gaussian_features,
                             to_gaussians.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Dict

import numpy as np
import torch

from . import _capi as C
from .block import GaussianBlock, Q8Weight, _Workspace
from .q8 import _ptr, _stream

REP_FIELDS = ("perturbe", "kernel", "scaling_bias", "opacity_bias", "lr_xyz", "lr_dc", "lr_opacity", "lr_scaling",
              "lr_rotation")
REP_DEFAULTS = (1.5, 0.0009, 0.004, 0.1, 1.0, 1.0, 1.0, 1.0, 0.1)  # src/weights.hpp:25-28


def read_native_export(path) -> Dict:
    """manifest.txt + weights.bin -> {"config": dict, "rep": tuple, "case": tuple or None, "tensors": {name: fp32
    array}, "qtensors": {name: (out, in, bits, group, uint8 blob)}}. Raises ValueError on a malformed export."""
    path = Path(path)
    lines = (path / "manifest.txt").read_text().splitlines()
    if not lines:
        raise ValueError(f"{path}/manifest.txt is empty")
    head = lines[0].split()
    if len(head) != 7 or head[0] != "decoders":
        raise ValueError("manifest.txt: the first line must be 'decoders dim heads oct gs cond per_anchor'")
    keys = ("dim", "heads", "oct_blocks", "gs_blocks", "cond", "per_anchor")
    out = {"config": dict(zip(keys, (int(v) for v in head[1:]))), "rep": REP_DEFAULTS, "case": None, "tensors": {},
           "qtensors": {}}
    data = np.fromfile(path / "weights.bin", dtype=np.uint8)
    for line in lines[1:]:
        f = line.split()
        if not f:
            continue
        if f[0] == "rep":
            out["rep"] = tuple(float(v) for v in f[1:10])
            continue
        if f[0] == "case":
            out["case"] = tuple(int(v) for v in f[1:4])
            continue
        if f[0] == "qtensor":
            name, o, i, bits, group, off, nb = f[1], *(int(v) for v in f[2:8])
            if off < 0 or nb < 0 or off + nb > data.size:
                raise ValueError(f"qtensor '{name}' lies outside weights.bin")
            out["qtensors"][name] = (o, i, bits, group, data[off:off + nb].copy())
            continue
        name, ndim = f[0], int(f[1])
        shape = tuple(int(v) for v in f[2:2 + ndim])
        off, nb = int(f[2 + ndim]), int(f[3 + ndim])
        if nb != int(np.prod(shape, dtype=np.int64)) * 4:
            raise ValueError(f"tensor '{name}' has a byte count that does not match its shape")
        if off < 0 or off + nb > data.size:
            raise ValueError(f"tensor '{name}' lies outside weights.bin")
        out["tensors"][name] = data[off:off + nb].view(np.float32).reshape(shape).copy()
    return out


def panels_to_q8(blob: np.ndarray, out: int, inp: int) -> np.ndarray:
    """8-bit, group-32 panel blob -> GGUF Q8_0 bytes [out * inp / 32 * 34]. Each 576-byte panel group holds 16 fp16
    scales, 16 fp16 minimums, then 32 rows of k x 16 columns of codes; a Q8_0 block is (scale, code - 128), exact
    when the minimum is -128 x scale."""
    panels, ng = (out + 15) // 16, inp // 32
    blob = np.asarray(blob, dtype=np.uint8)
    if blob.size != panels * ng * 576:
        raise ValueError("panel blob size does not match an 8-bit, group-32 matrix of this shape")
    g = blob.reshape(panels, ng, 576)
    scales = g[:, :, 0:32].copy().view(np.float16).reshape(panels, ng, 16)
    mins = g[:, :, 32:64].copy().view(np.float16).reshape(panels, ng, 16)
    if not np.array_equal(mins.astype(np.float32), np.float32(-128.0) * scales.astype(np.float32)):
        raise ValueError("panel minimums are not -128 x scale: not a Q8_0-derived 8-bit matrix")
    codes = g[:, :, 64:].reshape(panels, ng, 32, 16)                          # [p, g, k, c]
    q = (codes.astype(np.int16) - 128).astype(np.int8).transpose(0, 3, 1, 2)  # [p, c, g, k]
    q = q.reshape(panels * 16, ng, 32)[:out]
    d = scales.transpose(0, 2, 1).reshape(panels * 16, ng)[:out]              # [n, g]
    blocks = np.empty((out, ng, 34), np.uint8)
    blocks[:, :, 0:2] = d.copy().view(np.uint8).reshape(out, ng, 2)
    blocks[:, :, 2:] = q.view(np.uint8)
    return blocks.reshape(-1)


def _export_matrices(ex, device):
    """prefix, out, in -> Q8Weight of the export's matrix `prefix.weight` (+ `prefix.bias`) on `device`."""
    T, Q = ex["tensors"], ex["qtensors"]

    def q8w(prefix, out, inp):
        b = torch.from_numpy(T[prefix + ".bias"])
        if prefix + ".weight" in Q:
            o, i, bits, group, blob = Q[prefix + ".weight"]
            if (o, i, bits, group) != (out, inp, 8, 32):
                raise ValueError(f"{prefix}: only 8-bit, group-32 quantized matrices of shape ({out}, {inp})")
            q8 = torch.from_numpy(panels_to_q8(blob, out, inp)).to(device)
            return Q8Weight(q8, out, inp, b)
        return Q8Weight.from_float(torch.from_numpy(T[prefix + ".weight"]).to(device).reshape(out, inp), b)

    return q8w


class GaussianDecoder:
    """Decoders::gaussian_features + to_gaussians on one GPU (idol_b200_gs_decoder_*)."""

    def __init__(self, blocks, in_w, in_b, input_layer: Q8Weight, out_proj: Q8Weight, freqs, per_anchor: int,
                 perturbation, base_offset_scale: float, rep=REP_DEFAULTS):
        dev = input_layer.device

        def f32(t):
            return torch.as_tensor(t).detach().to(device=dev, dtype=torch.float32).contiguous()

        self.blocks = list(blocks)
        self.keep = (input_layer, out_proj)
        self.in_w, self.freqs, self.perturbation = f32(in_w), f32(freqs), f32(perturbation)
        self.in_b = None if in_b is None else f32(in_b)
        self.per_anchor, self.dim, self.device = per_anchor, input_layer.out, dev
        arr = (ctypes.c_void_p * max(1, len(self.blocks)))(*(b.handle for b in self.blocks))
        rep_c = (ctypes.c_float * 9)(*rep)
        h = ctypes.c_void_p()
        C.check(C.lib().idol_b200_gs_decoder_create(ctypes.cast(arr, ctypes.c_void_p), len(self.blocks),
                                                    _ptr(self.in_w), _ptr(self.in_b),
                                                    ctypes.c_void_p(input_layer.handle),
                                                    ctypes.c_void_p(out_proj.handle), _ptr(self.freqs),
                                                    self.freqs.numel(), per_anchor, _ptr(self.perturbation),
                                                    float(base_offset_scale), ctypes.cast(rep_c, ctypes.c_void_p),
                                                    ctypes.byref(h)))
        self.handle = h.value
        self.ws = _Workspace()

    @classmethod
    def from_native_export(cls, path, device, eps: float = 1e-6) -> "GaussianDecoder":
        """Reads an export (read_native_export) and uploads the Gaussian decoder's weights to `device` once.
        Q8_0-derived 8-bit matrices keep their Q8_0 values exactly; matrices the export holds as float32 are
        quantized to Q8_0 on the device (the reference multiplies those in fp32)."""
        ex = read_native_export(path)
        cfg, T = ex["config"], ex["tensors"]
        D, heads = cfg["dim"], cfg["heads"]
        device = torch.device(device)
        q8w = _export_matrices(ex, device)

        def vec(name):
            return torch.from_numpy(T[name])

        blocks = []
        for i in range(cfg["gs_blocks"]):
            p = f"gs.blocks.{i}."
            blocks.append(GaussianBlock(
                q8w(p + "self_attn.to_qkv", 3 * D, D), q8w(p + "self_attn.to_out", D, D),
                q8w(p + "cross_attn.to_q", D, D), q8w(p + "cross_attn.to_out", D, D),
                q8w(p + "mlp.mlp.0", 4 * D, D), q8w(p + "mlp.mlp.2", D, 4 * D),
                vec(p + "self_attn.q_rms_norm.gamma"), vec(p + "self_attn.k_rms_norm.gamma"),
                vec(p + "cross_attn.q_rms_norm.gamma"), vec(p + "cross_attn.k_rms_norm.gamma"),
                vec(p + "norm2.weight"), vec(p + "norm2.bias"),
                torch.from_numpy(T[p + "cross_attn.to_kv.weight"]).reshape(2 * D, cfg["cond"]),
                vec(p + "cross_attn.to_kv.bias"), heads, eps))
        G = cfg["per_anchor"]
        return cls(blocks, T["gs.in_proj.weight"].reshape(D, 3), T["gs.in_proj.bias"],
                   q8w("gs.input_layer", D, D), q8w("gs.out_proj", 15 * G, D), T["gs.pos_embedder.freqs"], G,
                   T["gs.points_offset_perturbation"], float(T["gs.base_offset_scale"].reshape(-1)[0]), ex["rep"])

    def features(self, points: torch.Tensor, cond: torch.Tensor) -> torch.Tensor:
        """points fp32 [rows, 3], cond fp32 [cond_rows, cond_dim] (CUDA) -> fp32 [rows, 15 per_anchor]."""
        points = points.to(device=self.device, dtype=torch.float32).contiguous()
        cond = cond.to(device=self.device, dtype=torch.float32).contiguous()
        rows = points.shape[0]
        out = torch.empty((rows, 15 * self.per_anchor), dtype=torch.float32, device=self.device)
        nbytes = int(C.lib().idol_b200_gs_decoder_workspace_bytes(ctypes.c_void_p(self.handle), rows,
                                                                  cond.shape[0]))
        ws = self.ws.get(nbytes, points.device)
        C.check(C.lib().idol_b200_gs_decoder_features(ctypes.c_void_p(self.handle), _ptr(points), rows, _ptr(cond),
                                                      cond.shape[0], _ptr(out), _ptr(ws), ws.numel(),
                                                      _stream(points.device)))
        return out

    def to_gaussians(self, anchors: torch.Tensor, features: torch.Tensor) -> Dict[str, torch.Tensor]:
        anchors = anchors.to(device=self.device, dtype=torch.float32).contiguous()
        features = features.to(device=self.device, dtype=torch.float32).contiguous()
        n = anchors.shape[0] * self.per_anchor
        out = {k: torch.empty((n, w), dtype=torch.float32, device=self.device)
               for k, w in (("xyz", 3), ("f_dc", 3), ("scale", 3), ("rotation", 4), ("opacity", 1))}
        C.check(C.lib().idol_b200_gs_to_gaussians(ctypes.c_void_p(self.handle), _ptr(anchors), anchors.shape[0],
                                                  _ptr(features), *(_ptr(out[k]) for k in
                                                                    ("xyz", "f_dc", "scale", "rotation", "opacity")),
                                                  _stream(anchors.device)))
        out["opacity"] = out["opacity"].reshape(-1)
        return out

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            try:
                C.lib().idol_b200_gs_decoder_free(ctypes.c_void_p(h))
            except Exception:
                pass
            self.handle = None


class OctreeSampler:
    """The host half of Decoders::sample_anchors: one instance per call, driven level by level with the logits of the
    cells it reports (same generator, order and arithmetic as the reference)."""

    def __init__(self, num_points: int, level: int, seed: int):
        h = ctypes.c_void_p()
        C.check(C.lib().idol_b200_oct_sampler_create(num_points, level, ctypes.c_uint64(seed), ctypes.byref(h)))
        self.handle, self.num_points = h.value, num_points

    def cells(self):
        """(number of cells to evaluate at the next level, their resolution); 0 cells once every level is done."""
        n, res = ctypes.c_int64(), ctypes.c_float()
        C.check(C.lib().idol_b200_oct_sampler_cells(ctypes.c_void_p(self.handle), ctypes.byref(n), ctypes.byref(res)))
        return n.value, res.value

    def centres(self) -> np.ndarray:
        n, _ = self.cells()
        out = np.empty((n, 3), np.float32)
        C.check(C.lib().idol_b200_oct_sampler_centres(ctypes.c_void_p(self.handle),
                                                      out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def step(self, logits) -> None:
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        C.check(C.lib().idol_b200_oct_sampler_step(ctypes.c_void_p(self.handle),
                                                   logits.ctypes.data_as(ctypes.c_void_p)))

    def points(self) -> np.ndarray:
        out = np.empty((self.num_points, 3), np.float32)
        C.check(C.lib().idol_b200_oct_sampler_points(ctypes.c_void_p(self.handle), out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def run(self, logits_fn) -> np.ndarray:
        """Every level with logits_fn(centres [n, 3], resolution) -> [n, 8], then the points."""
        while True:
            n, res = self.cells()
            if n == 0:
                return self.points()
            self.step(logits_fn(self.centres(), res))

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            try:
                C.lib().idol_b200_oct_sampler_free(ctypes.c_void_p(h))
            except Exception:
                pass
            self.handle = None


class OctreeDecoder:
    """Decoders::octree_logits + sample_anchors on one GPU (idol_b200_oct_*)."""

    def __init__(self, blocks, in_w, in_b, input_layer: Q8Weight, l1: Q8Weight, l2: Q8Weight, ada: Q8Weight,
                 out_proj: Q8Weight, freqs, level_freqs, heads: int, eps: float = 1e-6):
        """blocks: dicts of cq, co, ff1, ff2 (Q8Weight), kv_w [2D, cond_dim], kv_b [2D], cq_gamma, ck_gamma [D]."""
        dev = input_layer.device

        def f32(t):
            return torch.as_tensor(t).detach().to(device=dev, dtype=torch.float32).contiguous()

        self.keep = [input_layer, l1, l2, ada, out_proj]
        self.tensors = []
        self.block_handles = []
        for b in blocks:
            t = [f32(b[k]) for k in ("cq_gamma", "ck_gamma", "kv_w", "kv_b")]
            self.tensors += t
            self.keep += [b["cq"], b["co"], b["ff1"], b["ff2"]]
            h = ctypes.c_void_p()
            C.check(C.lib().idol_b200_oct_block_create(
                *(ctypes.c_void_p(b[k].handle) for k in ("cq", "co", "ff1", "ff2")), _ptr(t[0]), _ptr(t[1]),
                _ptr(t[2]), _ptr(t[3]), t[2].shape[1], heads, ctypes.byref(h)))
            self.block_handles.append(h.value)
        self.in_w, self.freqs, self.level_freqs = f32(in_w), f32(freqs), f32(level_freqs)
        self.in_b = None if in_b is None else f32(in_b)
        arr = (ctypes.c_void_p * max(1, len(self.block_handles)))(*self.block_handles)
        h = ctypes.c_void_p()
        C.check(C.lib().idol_b200_oct_decoder_create(
            ctypes.cast(arr, ctypes.c_void_p), len(self.block_handles), _ptr(self.in_w), _ptr(self.in_b),
            *(ctypes.c_void_p(m.handle) for m in (input_layer, l1, l2, ada, out_proj)), _ptr(self.freqs),
            self.freqs.numel(), _ptr(self.level_freqs), heads, float(eps), ctypes.byref(h)))
        self.handle, self.device = h.value, dev
        self.ws = _Workspace()

    @classmethod
    def from_native_export(cls, path, device, eps: float = 1e-6) -> "OctreeDecoder":
        ex = read_native_export(path)
        cfg, T = ex["config"], ex["tensors"]
        D, heads = cfg["dim"], cfg["heads"]
        q8w = _export_matrices(ex, torch.device(device))
        blocks = []
        for i in range(cfg["oct_blocks"]):
            p = f"oct.blocks.{i}."
            blocks.append({"cq": q8w(p + "cross_attn.to_q", D, D), "co": q8w(p + "cross_attn.to_out", D, D),
                           "ff1": q8w(p + "mlp.mlp.0", 4 * D, D), "ff2": q8w(p + "mlp.mlp.2", D, 4 * D),
                           "kv_w": T[p + "cross_attn.to_kv.weight"].reshape(2 * D, cfg["cond"]),
                           "kv_b": T[p + "cross_attn.to_kv.bias"],
                           "cq_gamma": T[p + "cross_attn.q_rms_norm.gamma"],
                           "ck_gamma": T[p + "cross_attn.k_rms_norm.gamma"]})
        return cls(blocks, T["oct.in_proj.weight"].reshape(D, 3), T["oct.in_proj.bias"],
                   q8w("oct.input_layer", D, D), q8w("oct.l_embedder.mlp.0", D, 256),
                   q8w("oct.l_embedder.mlp.2", D, D), q8w("oct.adaLN_modulation.1", 6 * D, D),
                   q8w("oct.out_proj", 8, D), T["oct.pos_embedder.freqs"], T["oct.l_embedder.freqs"], heads, eps)

    def _workspace(self, rows, cond_rows):
        n = int(C.lib().idol_b200_oct_decoder_workspace_bytes(ctypes.c_void_p(self.handle), rows, cond_rows))
        return self.ws.get(n, self.device)

    def logits(self, x, resolution: float, cond) -> torch.Tensor:
        """x: cell centres [rows, 3]; cond: [cond_rows, cond_dim] -> fp32 [rows, 8] on the device."""
        x = torch.as_tensor(x).to(device=self.device, dtype=torch.float32).contiguous()
        cond = torch.as_tensor(cond).to(device=self.device, dtype=torch.float32).contiguous()
        out = torch.empty((x.shape[0], 8), dtype=torch.float32, device=self.device)
        ws = self._workspace(x.shape[0], cond.shape[0])
        C.check(C.lib().idol_b200_oct_logits(ctypes.c_void_p(self.handle), _ptr(x), x.shape[0], float(resolution),
                                             _ptr(cond), cond.shape[0], _ptr(out), _ptr(ws), ws.numel(),
                                             _stream(self.device)))
        return out

    def sample_anchors(self, cond, num_points: int, level: int, seed: int) -> np.ndarray:
        """Decoders::sample_anchors -> host fp32 [num_points, 3]."""
        cond = torch.as_tensor(cond).to(device=self.device, dtype=torch.float32).contiguous()
        ws = self._workspace(num_points, cond.shape[0])
        out = np.empty((num_points, 3), np.float32)
        C.check(C.lib().idol_b200_oct_sample_anchors(ctypes.c_void_p(self.handle), _ptr(cond), cond.shape[0],
                                                     num_points, level, ctypes.c_uint64(seed),
                                                     out.ctypes.data_as(ctypes.c_void_p), _ptr(ws), ws.numel(),
                                                     _stream(self.device)))
        return out

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            try:
                C.lib().idol_b200_oct_decoder_free(ctypes.c_void_p(h))
                for b in self.block_handles:
                    C.lib().idol_b200_oct_block_free(ctypes.c_void_p(b))
            except Exception:
                pass
            self.handle = None


def decode(octree: OctreeDecoder, gaussian: GaussianDecoder, cond, num_gaussians: int, level: int, seed: int):
    """Decoders::decode (src/decoders.cpp:435-445): num_gaussians // per_anchor anchors (at least one) sampled from
    the latent, their features, then the activated Gaussians (a dict of device tensors)."""
    anchors = max(1, num_gaussians // gaussian.per_anchor)
    points = torch.from_numpy(octree.sample_anchors(cond, anchors, level, seed)).to(gaussian.device)
    cond = torch.as_tensor(cond).to(device=gaussian.device, dtype=torch.float32)
    return gaussian.to_gaussians(points, gaussian.features(points, cond))
