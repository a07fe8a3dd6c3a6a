"""Writes the committed golden vectors of tests/golden/ from the reference itself.

Run in a checkout where gguf-py 0.19.0 is importable and the reference's CPU kernels are built into
oracle/_ref/libidolref.so (``make -C oracle ref REF=<reference checkout>``):

    python tests/golden/make_golden.py

* q8_quant.npz   - fp32 weights (seeded normal plus hand-made edge rows: zeros, exact .5 ties, tiny and large values,
                   a single spike) and the bytes gguf.quantize(W, Q8_0) returns for them.
* gemm.npz       - per case: bf16-valued fp32 activations, Q8_0 weights from gguf, fp32 bias, and the reference's own
                   gemm_packed output (src/kernels.cpp float kernel through quantized_linear), including a column
                   window with a residual and GELU (the reference test's epilogue case, tests/test_kernels.cpp:138-155).
* ops.npz        - the reference's norm_rows / rms_heads / gelu_tanh / attention outputs on small seeded inputs.

The shapes follow the reference tests: tests/test_kernels.cpp:124-136,184-263 and tests/python/test_fused_packed.py:29-32.
"""
from __future__ import annotations

import sys
from pathlib import Path

import ctypes

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import gguf  # noqa: E402

from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent


def q8(w):
    return np.asarray(gguf.quantize(np.ascontiguousarray(w, np.float32), gguf.GGMLQuantizationType.Q8_0),
                      dtype=np.uint8).reshape(w.shape[0], -1)


def bf16(x):
    return O.f32_to_bf16_round(x)


def quant_cases():
    rng = np.random.default_rng(2024)
    w = rng.normal(0, 0.02, (24, 256)).astype(np.float32)
    w[0] = 0.0                                                  # all-zero blocks: d = 0, id = 0
    w[1, :32] = (np.arange(32) - 15.5).astype(np.float32)       # exact .5 ties after scaling
    w[2, :32] = np.float32(1e-30)                               # d far below fp16's subnormal range
    w[3, :32] = np.linspace(-3000, 3000, 32, dtype=np.float32)  # large magnitudes
    w[4, :32] = 0.0
    w[4, 7] = -1.0                                              # one spike: all other codes are 0
    w[5, :32] = np.float32(6.1e-5) * np.arange(32, dtype=np.float32)  # d in fp16's subnormal range
    w[6] = rng.normal(0, 1, 256).astype(np.float32) * np.float32(127.0)
    w[7, 32:64] = -w[7, 32:64]
    return w, q8(w)


def gemm_case(rng, m, n, k, window=None, gelu=False, residual=False):
    w = rng.normal(0, 0.25, (n, k)).astype(np.float32)
    q = q8(w)
    x = bf16(rng.normal(0, 1, (m, k)).astype(np.float32))
    b = rng.normal(0, 0.5, n).astype(np.float32)
    lin = O.RefLinear(q, b, n, k)
    n_off, cnt = window if window else (0, n)
    res = rng.normal(0, 0.5, (m, cnt)).astype(np.float32) if residual else None
    y = lin.gemm(x, n_off, cnt, res, gelu, mode=0)
    return dict(x=x, q8=q, bias=b, y=y, res=res if res is not None else np.zeros((0,), np.float32),
                meta=np.array([m, n, k, n_off, cnt, int(gelu), int(residual)], np.int64))


def main():
    if not O.have_ref():
        raise SystemExit("oracle/_ref/libidolref.so is missing: make -C oracle ref REF=<reference checkout>")
    O.ref_threads(1)

    w, q = quant_cases()
    np.savez_compressed(OUT / "q8_quant.npz", w=w, q8=q)

    rng = np.random.default_rng(144)
    cases = {}
    shapes = [(1, 7, 256), (41, 71, 256), (5, 33, 512), (19, 37, 128), (7, 20, 32), (5, 20, 64), (5, 20, 96),
              (3, 130, 224), (33, 96, 1024)]
    for i, (m, n, k) in enumerate(shapes):
        cases[f"c{i}"] = gemm_case(rng, m, n, k)
    cases["win"] = gemm_case(rng, 6, 37, 64, window=(16, 21), gelu=True, residual=True)
    cases["win2"] = gemm_case(rng, 19, 64, 128, window=(32, 32), gelu=False, residual=True)
    flat = {f"{name}/{key}": val for name, case in cases.items() for key, val in case.items()}
    np.savez_compressed(OUT / "gemm.npz", **flat)

    R = O.ref()
    rng = np.random.default_rng(7)
    rows, dim = 9, 256
    x = rng.normal(0, 2, (rows, dim)).astype(np.float32)
    g = rng.normal(1, 0.2, dim).astype(np.float32)
    bt = rng.normal(0, 0.2, dim).astype(np.float32)
    sh = rng.normal(0, 0.2, dim).astype(np.float32)
    sc = rng.normal(0, 0.2, dim).astype(np.float32)
    ln_plain = np.empty_like(x)
    R.ref_norm_rows(O._ptr(x), O._ptr(ln_plain), rows, dim, 1e-6, None, None, None, None)
    ln_affine = np.empty_like(x)
    R.ref_norm_rows(O._ptr(x), O._ptr(ln_affine), rows, dim, 1e-6, O._ptr(g), O._ptr(bt), None, None)
    ln_ada = np.empty_like(x)
    R.ref_norm_rows(O._ptr(x), O._ptr(ln_ada), rows, dim, 1e-5, None, None, O._ptr(sh), O._ptr(sc))
    heads, hd = 4, 64
    qk = rng.normal(0, 1, (rows, 3 * dim)).astype(np.float32)
    gam = rng.normal(1, 0.1, dim).astype(np.float32)
    rms = qk.copy()
    R.ref_rms_heads(O._ptr(rms), rows, 3 * dim, heads, hd, O._ptr(gam))
    gt = rng.normal(0, 2, 1000).astype(np.float32)
    gt_out = gt.copy()
    R.ref_gelu_tanh(O._ptr(gt_out), gt.size)
    lq, lk = 37, 53
    # bf16-representable inputs: the GPU path takes q, k and v in bf16, so the comparison measures the kernel alone
    aq = bf16(rng.normal(0, 1, (lq, 3 * dim)).astype(np.float32))
    ak = bf16(rng.normal(0, 1, (lk, 2 * dim)).astype(np.float32))
    # k = ak[:, :dim] and v = the same rows shifted by dim columns, as the decoders pass kv and kv + D
    att = np.empty((lq, dim), np.float32)
    vptr = ctypes.cast(ak.ctypes.data + 4 * dim, O._f32p)
    R.ref_attention(O._ptr(aq), lq, 3 * dim, O._ptr(ak), vptr, lk, 2 * dim, heads, hd, O._ptr(att), dim)
    np.savez_compressed(OUT / "ops.npz", x=x, gamma=g, beta=bt, shift=sh, scale=sc, ln_plain=ln_plain,
                        ln_affine=ln_affine, ln_ada=ln_ada, qk=qk, qk_gamma=gam, rms=rms, gelu_in=gt,
                        gelu_out=gt_out, att_q=aq, att_kv=ak, att_out=att,
                        meta=np.array([rows, dim, heads, hd, lq, lk], np.int64))
    for p in sorted(OUT.glob("*.npz")):
        print(f"{p.name}: {p.stat().st_size} bytes")


if __name__ == "__main__":
    main()
