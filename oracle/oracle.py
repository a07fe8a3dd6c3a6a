"""ctypes front end for the CPU checkers (test infrastructure, never the product).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` / ``--impl reference`` legs import this
module. It wraps two libraries built by ``oracle/Makefile``:

* ``liboracle.so`` - the C restatement of the reference's Q8_0 path (q8_oracle.c; each function cites the reference
  file:line it follows).
* ``_ref/libidolref.so`` - the reference's own CPU kernels (src/kernels.cpp, src/weights.cpp, src/decoders.cpp)
  compiled from the reference tree. Present only where that tree was available at build time; ``have_ref()`` says so.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ACT_NONE, ACT_GELU_ERF, ACT_GELU_TANH, ACT_SILU = 0, 1, 2, 3

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_lib = None
_ref = None


def _ptr(a, kind=_f32p):
    return None if a is None else a.ctypes.data_as(kind)


def lib():
    global _lib
    if _lib is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            raise RuntimeError(f"{path} is missing: run `make -C oracle`")
        L = ctypes.CDLL(str(path))
        L.orc_q8_quantize.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, _u8p]
        L.orc_q8_dequantize.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int64, _f32p]
        L.orc_q4_0_dequantize.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int64, _f32p]
        L.orc_q4_0_to_q8.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int64, _u8p]
        L.orc_q4_k_dequantize.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int64, _f32p]
        L.orc_panel_blob_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
        L.orc_panel_blob_bytes.restype = ctypes.c_int64
        L.orc_q8_to_panels.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, _u8p]
        L.orc_gemm_q8.argtypes = [_f32p, ctypes.c_int, _u8p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, _f32p, ctypes.c_int, _f32p]
        L.orc_gemm_q8_int8act.argtypes = L.orc_gemm_q8.argtypes
        L.orc_quantize_activations.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int8),
                                               _f32p, ctypes.POINTER(ctypes.c_int32)]
        L.orc_activate.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int]
        L.orc_norm_rows.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p, _f32p, _f32p,
                                    _f32p]
        L.orc_rms_heads.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_attention.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int]
        L.orc_gaussian_heads.argtypes = [_f32p, ctypes.c_int64, _f32p]
        L.orc_pos_embed.argtypes = [_f32p, ctypes.c_int64, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_level_embed.argtypes = [ctypes.c_float, _f32p, _f32p]
        L.orc_to_gaussians.argtypes = [_f32p, ctypes.c_int64, _f32p, ctypes.c_int, _f32p, ctypes.c_float, _f32p,
                                       _f32p, _f32p, _f32p, _f32p, _f32p]
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f32.restype = ctypes.c_float
        for name in ("orc_gelu_erf", "orc_gelu_tanh", "orc_silu"):
            getattr(L, name).argtypes = [ctypes.c_float]
            getattr(L, name).restype = ctypes.c_float
        _lib = L
    return _lib


def have_ref() -> bool:
    return (HERE / "_ref" / "libidolref.so").exists()


def ref():
    global _ref
    if _ref is None:
        path = HERE / "_ref" / "libidolref.so"
        if not path.exists():
            raise RuntimeError(f"{path} is missing: run `make -C oracle ref REF=<reference checkout>`")
        R = ctypes.CDLL(str(path))
        R.ref_last_error.restype = ctypes.c_char_p
        R.ref_set_threads.argtypes = [ctypes.c_int]
        R.ref_max_threads.restype = ctypes.c_int
        R.ref_q8_linear_create.argtypes = [_u8p, _f32p, ctypes.c_int, ctypes.c_int]
        R.ref_q8_linear_create.restype = ctypes.c_void_p
        R.ref_blob_linear_create.argtypes = [_u8p, ctypes.c_int64, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int]
        R.ref_blob_linear_create.restype = ctypes.c_void_p
        R.ref_linear_free.argtypes = [ctypes.c_void_p]
        R.ref_gemm.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int,
                               _f32p, ctypes.c_int]
        R.ref_dequantize.argtypes = [ctypes.c_void_p, _f32p]
        R.ref_norm_rows.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p, _f32p, _f32p,
                                    _f32p]
        R.ref_layer_norm.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p]
        R.ref_rms_heads.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        R.ref_gelu_tanh.argtypes = [_f32p, ctypes.c_int64]
        R.ref_silu.argtypes = [ctypes.c_float]
        R.ref_silu.restype = ctypes.c_float
        R.ref_gelu_scalar.argtypes = [ctypes.c_float]
        R.ref_gelu_scalar.restype = ctypes.c_float
        R.ref_attention.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int]
        R.ref_decoders_open.argtypes = [ctypes.c_char_p]
        R.ref_decoders_open.restype = ctypes.c_void_p
        R.ref_decoders_free.argtypes = [ctypes.c_void_p]
        R.ref_gaussian_features.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, _f32p, ctypes.c_int, _f32p,
                                            ctypes.c_int]
        R.ref_to_gaussians.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, _f32p, _f32p, _f32p, _f32p, _f32p,
                                       _f32p]
        R.ref_octree_logits.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_float, _f32p, ctypes.c_int,
                                        _f32p, ctypes.c_int]
        R.ref_sample_anchors.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_uint64, _f32p, ctypes.c_int]
        R.ref_sample_anchors.restype = ctypes.c_int
        _ref = R
    return _ref


# ---------------------------------------------------------------------------------------------------- the restatement
def c32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def q8_quantize(w: np.ndarray) -> np.ndarray:
    """fp32 [rows, cols] -> Q8_0 bytes [rows, cols/32*34] with gguf-py 0.19.0 semantics."""
    w = c32(w)
    rows, cols = w.shape
    out = np.empty((rows, cols // 32 * 34), np.uint8)
    lib().orc_q8_quantize(_ptr(w), rows, cols, _ptr(out, _u8p))
    return out


def q8_dequantize(q8: np.ndarray, rows: int, cols: int) -> np.ndarray:
    q8 = np.ascontiguousarray(q8, dtype=np.uint8)
    out = np.empty((rows, cols), np.float32)
    lib().orc_q8_dequantize(_ptr(q8, _u8p), rows, cols, _ptr(out))
    return out


def q4_0_dequantize(q4: np.ndarray, rows: int, cols: int) -> np.ndarray:
    q4 = np.ascontiguousarray(q4, dtype=np.uint8)
    out = np.empty((rows, cols), np.float32)
    lib().orc_q4_0_dequantize(_ptr(q4, _u8p), rows, cols, _ptr(out))
    return out


def q4_k_dequantize(q4k: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """GGUF Q4_K bytes -> fp32 [rows, cols] (the reference's expansion, tools/idol_packed.py:41-54)."""
    q4k = np.ascontiguousarray(q4k, dtype=np.uint8).reshape(-1)
    assert q4k.size == rows * (cols // 256) * 144 and cols % 256 == 0
    out = np.empty((rows, cols), np.float32)
    lib().orc_q4_k_dequantize(_ptr(q4k, _u8p), rows, cols, _ptr(out))
    return out


def q4_0_to_q8(q4: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Q4_0 bytes -> the Q8_0 bytes of the same weights (exact)."""
    q4 = np.ascontiguousarray(q4, dtype=np.uint8)
    out = np.empty(rows * (cols // 32) * 34, np.uint8)
    lib().orc_q4_0_to_q8(_ptr(q4, _u8p), rows, cols, _ptr(out, _u8p))
    return out


def q8_to_panels(q8: np.ndarray, out: int, inp: int) -> np.ndarray:
    q8 = np.ascontiguousarray(q8, dtype=np.uint8)
    blob = np.empty(lib().orc_panel_blob_bytes(out, inp), np.uint8)
    rc = lib().orc_q8_to_panels(_ptr(q8, _u8p), out, inp, _ptr(blob, _u8p))
    if rc != 0:
        raise ValueError(f"Q8_0 -> panel conversion failed ({rc})")
    return blob


def gemm_q8(a, q8, bias, N, K, n_offset=0, n=None, residual=None, act=ACT_NONE):
    """C = A . W[n_offset:n_offset+n]^T + bias (+ residual) (-> act), the reference float kernel's summation order."""
    a = c32(a)
    m = a.shape[0]
    n = N - n_offset if n is None else n
    q8 = np.ascontiguousarray(q8, dtype=np.uint8)
    bias = None if bias is None else c32(bias)
    residual = None if residual is None else c32(residual)
    c = np.empty((m, n), np.float32)
    lib().orc_gemm_q8(_ptr(a), m, _ptr(q8, _u8p), _ptr(bias), N, K, n_offset, n, _ptr(residual), act, _ptr(c))
    return c


def gemm_q8_int8act(a, q8, bias, N, K, n_offset=0, n=None, residual=None, act=ACT_NONE):
    """The reference's integer-activation kernel (src/kernels.cpp:368-479): activations quantized per (row, 32-group)
    to int8, integer dot products per group, the group's float update in the reference's order."""
    a = c32(a)
    m = a.shape[0]
    n = N - n_offset if n is None else n
    q8 = np.ascontiguousarray(q8, dtype=np.uint8)
    bias = None if bias is None else c32(bias)
    residual = None if residual is None else c32(residual)
    c = np.empty((m, n), np.float32)
    lib().orc_gemm_q8_int8act(_ptr(a), m, _ptr(q8, _u8p), _ptr(bias), N, K, n_offset, n, _ptr(residual), act,
                              _ptr(c))
    return c


def quantize_activations(a):
    """(qa int8 [m, K], scale fp32 [m, K/32], qsum int32 [m, K/32]) as src/kernels.cpp:368-402."""
    a = c32(a)
    m, K = a.shape
    qa = np.empty((m, K), np.int8)
    sc = np.empty((m, K // 32), np.float32)
    qs = np.empty((m, K // 32), np.int32)
    lib().orc_quantize_activations(_ptr(a), m, K, qa.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)), _ptr(sc),
                                   qs.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    return qa, sc, qs


def activate(x, act):
    x = c32(x).copy()
    lib().orc_activate(_ptr(x), x.size, act)
    return x


def norm_rows(x, eps, gamma=None, beta=None, shift=None, scale=None):
    x = c32(x)
    rows, dim = x.shape
    y = np.empty_like(x)
    lib().orc_norm_rows(_ptr(x), _ptr(y), rows, dim, eps, _ptr(None if gamma is None else c32(gamma)),
                        _ptr(None if beta is None else c32(beta)), _ptr(None if shift is None else c32(shift)),
                        _ptr(None if scale is None else c32(scale)))
    return y


def rms_heads(x, heads, hd, gamma, col0=0, ld=None):
    """Per-head L2 norm over columns [col0, col0 + heads*hd) of each row; returns a copy."""
    x = c32(x).copy()
    rows = x.shape[0]
    ld = x.shape[1] if ld is None else ld
    gamma = c32(gamma)
    base = x.ctypes.data + 4 * col0
    lib().orc_rms_heads(ctypes.cast(base, _f32p), rows, ld, heads, hd, _ptr(gamma))
    return x


def attention(q, k, v, heads, head_dim):
    """q [lq, >=dim], k/v [lk, >=dim] (rows of their own strides) -> out [lq, dim]."""
    q, k, v = c32(q), c32(k), c32(v)
    dim = heads * head_dim
    out = np.empty((q.shape[0], dim), np.float32)
    lib().orc_attention(_ptr(q), q.shape[0], q.shape[1], _ptr(k), _ptr(v), k.shape[0], k.shape[1], heads, head_dim,
                        _ptr(out), dim)
    return out


def gaussian_heads(raw):
    raw = c32(raw)
    out = np.empty_like(raw)
    lib().orc_gaussian_heads(_ptr(raw), raw.shape[0], _ptr(out))
    return out


def f32_to_bf16_round(x):
    """fp32 values rounded to bf16 (round to nearest even), returned as fp32."""
    x = c32(x)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    return r.astype(np.uint32).view(np.float32)


# ------------------------------------------------------------------------------------------- composed block oracles
def block_forward(x, layers, heads, eps=1e-6, images=1, bf16_stream=False):
    """The denoiser-style block of the scope table (src/decoders.cpp:296-313 without the cross-attention):
    LN -> QKV -> rms q,k -> self-attention per image -> out + res -> LN -> ff1 -> gelu_tanh -> ff2 + res.
    x: [images * L, D] fp32; layers: dict of (q8, bias, N, K) for qkv/out/ff1/ff2 plus q_gamma/k_gamma.
    bf16_stream: the residual stream is stored in bf16 (rounded after each residual sublayer)."""
    rnd = f32_to_bf16_round if bf16_stream else (lambda v: v)
    x = c32(x)
    rows, D = x.shape
    hd = D // heads
    L = rows // images
    h = norm_rows(x, eps)
    qkv = gemm_q8(h, *layers["qkv"])
    qkv = rms_heads(qkv, heads, hd, layers["q_gamma"], col0=0)
    qkv = rms_heads(qkv, heads, hd, layers["k_gamma"], col0=D)
    a = np.empty((rows, D), np.float32)
    for i in range(images):
        blk = qkv[i * L:(i + 1) * L]
        a[i * L:(i + 1) * L] = attention(blk[:, :D], np.ascontiguousarray(blk[:, D:2 * D]),
                                         np.ascontiguousarray(blk[:, 2 * D:]), heads, hd)
    x = rnd(gemm_q8(a, *layers["out"], residual=x))
    h = norm_rows(x, eps)
    f = gemm_q8(h, *layers["ff1"], act=ACT_GELU_TANH)
    return rnd(gemm_q8(f, *layers["ff2"], residual=x))


def gs_block_forward(x, cond, layers, heads, eps=1e-6, images=1, bf16_stream=False):
    """The Gaussian decoder's block (src/decoders.cpp:296-313), composed from the pinned functions in the reference's
    order: LN -> QKV -> rms q,k -> self-attention -> out + res; LN * gamma2 + beta2 -> cross-attention
    (src/decoders.cpp:232-240: q = h Wq, rms q; kv = cond Wkv + b with the dense fp32 to_kv, rms k; attention of the
    image's rows over its cond rows) -> out + res; LN -> ff1 -> gelu_tanh -> ff2 + res.
    x: [images * L, D]; cond: [images * Lc, cond_dim] fp32; layers: the block's dict plus cq, co (q8, bias, N, K),
    kv_w [2D, cond_dim], kv_b [2D], cq_gamma, ck_gamma, norm2_gamma, norm2_beta. bf16_stream: the residual stream
    is stored in bf16, so x is rounded to bf16 after each residual sublayer (as a bf16 caller's stream is)."""
    rnd = f32_to_bf16_round if bf16_stream else (lambda v: v)
    x = c32(x)
    cond = c32(cond)
    rows, D = x.shape
    hd = D // heads
    L = rows // images
    Lc = cond.shape[0] // images
    h = norm_rows(x, eps)
    qkv = gemm_q8(h, *layers["qkv"])
    qkv = rms_heads(qkv, heads, hd, layers["q_gamma"], col0=0)
    qkv = rms_heads(qkv, heads, hd, layers["k_gamma"], col0=D)
    a = np.empty((rows, D), np.float32)
    for i in range(images):
        blk = qkv[i * L:(i + 1) * L]
        a[i * L:(i + 1) * L] = attention(blk[:, :D], np.ascontiguousarray(blk[:, D:2 * D]),
                                         np.ascontiguousarray(blk[:, 2 * D:]), heads, hd)
    x = rnd(gemm_q8(a, *layers["out"], residual=x))
    h = norm_rows(x, eps, layers["norm2_gamma"], layers["norm2_beta"])
    q = rms_heads(gemm_q8(h, *layers["cq"]), heads, hd, layers["cq_gamma"], col0=0)
    kv = (cond.astype(np.float64) @ c32(layers["kv_w"]).astype(np.float64).T + layers["kv_b"]).astype(np.float32)
    kv = rms_heads(kv, heads, hd, layers["ck_gamma"], col0=0)
    for i in range(images):
        kvi = kv[i * Lc:(i + 1) * Lc]
        a[i * L:(i + 1) * L] = attention(q[i * L:(i + 1) * L], np.ascontiguousarray(kvi[:, :D]),
                                         np.ascontiguousarray(kvi[:, D:]), heads, hd)
    x = rnd(gemm_q8(a, *layers["co"], residual=x))
    h = norm_rows(x, eps)
    f = gemm_q8(h, *layers["ff1"], act=ACT_GELU_TANH)
    return rnd(gemm_q8(f, *layers["ff2"], residual=x))


# The reference's Representation defaults (src/weights.hpp:25-28), in orc_to_gaussians' order.
REPRESENTATION = dict(perturbe=1.5, kernel=0.0009, scaling_bias=0.004, opacity_bias=0.1, lr_xyz=1.0, lr_dc=1.0,
                      lr_opacity=1.0, lr_scaling=1.0, lr_rotation=0.1)


def pos_embed(points, freqs, dim):
    points, freqs = c32(points), c32(freqs)
    out = np.empty((points.shape[0], dim), np.float32)
    lib().orc_pos_embed(_ptr(points), points.shape[0], _ptr(freqs), freqs.size, dim, _ptr(out))
    return out


def to_gaussians(anchors, features, per_anchor, perturbation, base_offset_scale, rep=None):
    """Decoders::to_gaussians (src/decoders.cpp:393-433) -> dict of xyz, f_dc, scale, rotation, opacity."""
    rep = dict(REPRESENTATION, **(rep or {}))
    r = c32([rep[k] for k in REPRESENTATION])
    anchors, features, perturbation = c32(anchors), c32(features), c32(perturbation)
    n = anchors.shape[0] * per_anchor
    out = {k: np.empty((n, w), np.float32) for k, w in (("xyz", 3), ("f_dc", 3), ("scale", 3), ("rotation", 4),
                                                         ("opacity", 1))}
    lib().orc_to_gaussians(_ptr(anchors), anchors.shape[0], _ptr(features), per_anchor, _ptr(perturbation),
                           float(base_offset_scale), _ptr(r), *(_ptr(out[k]) for k in
                                                                ("xyz", "f_dc", "scale", "rotation", "opacity")))
    out["opacity"] = out["opacity"].reshape(-1)
    return out


def gaussian_features(points, cond, dec, heads, eps=1e-6):
    """Decoders::Impl::gaussian_features (src/decoders.cpp:284-316) for one image: pos_embed + in_proj (dense fp32,
    K = 3) as its residual -> input_layer -> the blocks -> LN (eps 1e-5) -> out_proj. dec: in_w [D, 3], in_b [D],
    input (q8, bias, N, K), blocks (list of gs_block_forward layer dicts), out (q8, bias, N, K), freqs."""
    points = c32(points)
    D = dec["in_w"].shape[0]
    h = pos_embed(points, dec["freqs"], D)
    x = (points @ c32(dec["in_w"]).T + dec["in_b"] + h).astype(np.float32)
    x = gemm_q8(x, *dec["input"])
    for layers in dec["blocks"]:
        x = gs_block_forward(x, cond, layers, heads, eps)
    h = norm_rows(x, 1e-5)
    return gemm_q8(h, *dec["out"])


def level_embed(resolution, freqs):
    out = np.empty(256, np.float32)
    lib().orc_level_embed(float(resolution), _ptr(c32(freqs)), _ptr(out))
    return out


def octree_logits(x, resolution, cond, dec, heads, eps=1e-6):
    """Decoders::Impl::octree_logits (src/decoders.cpp:242-282): pos_embed + in_proj (dense fp32, K = 3) ->
    input_layer; the level embedding -> l1 -> SiLU -> l2 -> SiLU -> adaLN modulation (shift, scale, gate for the
    attention and the MLP half); per block: LN * (1 + scale_a) + shift_a -> cross-attention -> to_out, added with
    gate_a; LN * (1 + scale_m) + shift_m -> ff1 -> gelu_tanh -> ff2, added with gate_m; LN (eps 1e-5) -> out_proj (8
    logits). dec: in_w [D, 3], in_b, input, l1, l2, ada, out (q8, bias, N, K), freqs, level_freqs, blocks (dicts of
    cq, co, ff1, ff2, kv_w, kv_b, cq_gamma, ck_gamma)."""
    x, cond = c32(x), c32(cond)
    D = dec["in_w"].shape[0]
    hd = D // heads
    h = pos_embed(x, dec["freqs"], D)
    X = (x @ c32(dec["in_w"]).T + dec["in_b"] + h).astype(np.float32)
    X = gemm_q8(X, *dec["input"])
    emb = level_embed(resolution, dec["level_freqs"]).reshape(1, 256)
    l1 = activate(gemm_q8(emb, *dec["l1"]), ACT_SILU)
    l2 = activate(gemm_q8(l1, *dec["l2"]), ACT_SILU)
    mod = gemm_q8(l2, *dec["ada"]).reshape(6, D)
    shift_a, scale_a, gate_a, shift_m, scale_m, gate_m = mod
    for L in dec["blocks"]:
        h = norm_rows(X, eps, shift=shift_a, scale=scale_a)
        q = rms_heads(gemm_q8(h, *L["cq"]), heads, hd, L["cq_gamma"], col0=0)
        kv = (cond.astype(np.float64) @ c32(L["kv_w"]).astype(np.float64).T + L["kv_b"]).astype(np.float32)
        kv = rms_heads(kv, heads, hd, L["ck_gamma"], col0=0)
        a = attention(q, np.ascontiguousarray(kv[:, :D]), np.ascontiguousarray(kv[:, D:]), heads, hd)
        X = (X + gemm_q8(a, *L["co"]) * gate_a).astype(np.float32)
        h = norm_rows(X, eps, shift=shift_m, scale=scale_m)
        f = gemm_q8(h, *L["ff1"], act=ACT_GELU_TANH)
        X = (X + gemm_q8(f, *L["ff2"]) * gate_m).astype(np.float32)
    return gemm_q8(norm_rows(X, 1e-5), *dec["out"])


def gaussian_mlp(x, layers):
    """Synthetic Gaussian MLP: 128 -> 512 (SiLU) -> 512 (SiLU) -> 14, then the activated heads."""
    h = gemm_q8(x, *layers[0], act=ACT_SILU)
    h = gemm_q8(h, *layers[1], act=ACT_SILU)
    raw = gemm_q8(h, *layers[2])
    return raw, gaussian_heads(raw)


# --------------------------------------------------------------------------------------- the reference, as compiled
class RefLinear:
    """The reference's own PackedLinear built from Q8_0 blocks (tools/gguf_to_decoder.py -> quantized_linear)."""

    def __init__(self, q8, bias, out, inp):
        self.q8 = np.ascontiguousarray(q8, dtype=np.uint8)
        self.bias = c32(bias if bias is not None else np.zeros(out, np.float32))
        self.out, self.inp = out, inp
        self.h = ref().ref_q8_linear_create(_ptr(self.q8, _u8p), _ptr(self.bias), out, inp)
        if not self.h:
            raise ValueError(ref().ref_last_error().decode())

    def gemm(self, a, n_offset=0, n=None, residual=None, gelu=False, mode=0):
        a = c32(a)
        n = self.out - n_offset if n is None else n
        c = np.empty((a.shape[0], n), np.float32)
        ref().ref_gemm(self.h, _ptr(a), a.shape[0], n_offset, n, _ptr(None if residual is None else c32(residual)),
                       int(gelu), _ptr(c), mode)
        return c

    def dequantize(self):
        w = np.empty((self.out, self.inp), np.float32)
        ref().ref_dequantize(self.h, _ptr(w))
        return w

    def __del__(self):
        if getattr(self, "h", None):
            ref().ref_linear_free(self.h)
            self.h = None


class RefBlock:
    """The config-3/5 block composed of the reference's own CPU functions as compiled into _ref (test infrastructure:
    the timed CPU baseline of the denoiser stack, checked against block_forward): norm_rows (src/decoders.cpp:23-42),
    gemm_packed with the float kernel (src/kernels.cpp:552-565), rms_heads (src/decoders.cpp:74-86), attention
    (src/kernels.cpp:737-746) and gelu_tanh (src/decoders.cpp:55-71), in the order of src/decoders.cpp:296-313 without
    the cross-attention. `layers` as for block_forward."""

    def __init__(self, layers, heads, eps=1e-6):
        self.lin = {n: RefLinear(*layers[n]) for n in ("qkv", "out", "ff1", "ff2")}
        self.qg, self.kg = c32(layers["q_gamma"]), c32(layers["k_gamma"])
        self.heads, self.eps = heads, eps

    def forward_(self, x, images=1, mode=0):
        """In place on x: [images * L, D] fp32 C-contiguous. mode 0: the float GEMM kernel (production), 1: the
        integer-activation kernel."""
        R = ref()
        rows, D = x.shape
        hd, L = D // self.heads, rows // images
        h = np.empty_like(x)
        R.ref_norm_rows(_ptr(x), _ptr(h), rows, D, self.eps, None, None, None, None)
        qkv = self.lin["qkv"].gemm(h, mode=mode)
        R.ref_rms_heads(_ptr(qkv), rows, 3 * D, self.heads, hd, _ptr(self.qg))
        R.ref_rms_heads(ctypes.cast(qkv.ctypes.data + 4 * D, _f32p), rows, 3 * D, self.heads, hd, _ptr(self.kg))
        a = np.empty((rows, D), np.float32)
        for i in range(images):
            base = qkv.ctypes.data + 4 * i * L * 3 * D
            R.ref_attention(ctypes.cast(base, _f32p), L, 3 * D, ctypes.cast(base + 4 * D, _f32p),
                            ctypes.cast(base + 8 * D, _f32p), L, 3 * D, self.heads, hd,
                            ctypes.cast(a.ctypes.data + 4 * i * L * D, _f32p), D)
        x[:] = self.lin["out"].gemm(a, residual=x, mode=mode)
        R.ref_norm_rows(_ptr(x), _ptr(h), rows, D, self.eps, None, None, None, None)
        f = self.lin["ff1"].gemm(h, mode=mode)
        R.ref_gelu_tanh(_ptr(f), f.size)
        x[:] = self.lin["ff2"].gemm(f, residual=x, mode=mode)
        return x


def ref_threads(n=None):
    if n is None:
        n = os.cpu_count() or 1
    ref().ref_set_threads(int(n))
    return int(n)


class RefDecoders:
    """The reference's Decoders (include/idol/decoders.hpp) loaded from a native export directory."""

    def __init__(self, path):
        self.h = ref().ref_decoders_open(str(path).encode())
        if not self.h:
            raise ValueError(ref().ref_last_error().decode())

    def gaussian_features(self, points, cond, outs, mode=0):
        """mode 0: the float kernel production forces (tools/idol_generate.py:356); 1: the AVX-VNNI kernel."""
        points, cond = c32(points), c32(cond)
        out = np.empty((points.shape[0], outs), np.float32)
        ref().ref_gaussian_features(self.h, _ptr(points), points.shape[0], _ptr(cond), cond.shape[0], _ptr(out),
                                    mode)
        return out

    def octree_logits(self, x, resolution, cond, mode=0):
        x, cond = c32(x), c32(cond)
        out = np.empty((x.shape[0], 8), np.float32)
        ref().ref_octree_logits(self.h, _ptr(x), x.shape[0], float(resolution), _ptr(cond), cond.shape[0], _ptr(out),
                                mode)
        return out

    def sample_anchors(self, cond, num_points, level, seed, mode=0):
        cond = c32(cond)
        out = np.empty((num_points, 3), np.float32)
        n = ref().ref_sample_anchors(self.h, _ptr(cond), cond.shape[0], num_points, level, seed, _ptr(out), mode)
        if n < 0:
            raise ValueError(ref().ref_last_error().decode())
        return out

    def to_gaussians(self, anchors, features, per_anchor):
        anchors, features = c32(anchors), c32(features)
        n = anchors.shape[0] * per_anchor
        out = {k: np.empty((n, w), np.float32) for k, w in (("xyz", 3), ("f_dc", 3), ("scale", 3), ("rotation", 4),
                                                             ("opacity", 1))}
        ref().ref_to_gaussians(self.h, _ptr(anchors), anchors.shape[0], _ptr(features),
                               *(_ptr(out[k]) for k in ("xyz", "f_dc", "scale", "rotation", "opacity")))
        out["opacity"] = out["opacity"].reshape(-1)
        return out

    def __del__(self):
        if getattr(self, "h", None):
            ref().ref_decoders_free(self.h)
            self.h = None
