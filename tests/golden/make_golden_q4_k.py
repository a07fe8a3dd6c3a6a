"""Writes tests/golden/q4_k.npz, the GGUF Q4_K (kind 44) golden vectors, from gguf-py 0.19.0 and the reference itself.

Run in a checkout where gguf-py is importable and the reference checkout is given by IDOL_REFERENCE:

    IDOL_REFERENCE=<reference checkout> python tests/golden/make_golden_q4_k.py

gguf-py 0.19.0 has no Q4_K encoder, so the bytes are seeded random super-blocks (fp16 d and dmin of weight-like
magnitude, random 6-bit scale / min bytes and codes) plus edge rows: all zero; subnormal d and dmin; negative d and
dmin; every scale, min and code byte 0xFF; the largest finite fp16 d. q4_k.npz holds the bytes, gguf.dequantize of
them, and the reference's own expansion (tools/idol_packed.py PackedLinear.dequantize, the path its unfused layers
take).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

import gguf

OUT = Path(__file__).resolve().parent
ROWS, COLS = 21, 768


def q4_k_cases(rows=ROWS, cols=COLS, seed=44):
    rng = np.random.default_rng(seed)
    nsb = cols // 256
    blocks = rng.integers(0, 256, size=(rows, nsb, 144), dtype=np.uint8)
    d = np.abs(rng.normal(0, 2e-4, (rows, nsb))).astype(np.float16)
    dmin = np.abs(rng.normal(0, 2e-3, (rows, nsb))).astype(np.float16)
    blocks[:, :, 0:2] = d.view(np.uint8).reshape(rows, nsb, 2)
    blocks[:, :, 2:4] = dmin.view(np.uint8).reshape(rows, nsb, 2)
    blocks[0] = 0                                                    # all zero
    blocks[1, :, 0:4] = np.array([1, 0, 1, 0], np.uint8)             # subnormal d and dmin (2^-24)
    neg = np.array([-3e-4, -1e-3], np.float16).view(np.uint8)        # negative d and dmin
    blocks[2, :, 0:4] = neg
    blocks[3, :, 4:] = 0xFF                                          # scales, mins and codes all ones
    blocks[4, :, 0:2] = np.array([65504.0], np.float16).view(np.uint8)  # the largest finite d
    return blocks.reshape(-1)


def main():
    ref = os.environ.get("IDOL_REFERENCE")
    if not ref or not (Path(ref) / "tools" / "idol_packed.py").exists():
        raise SystemExit("set IDOL_REFERENCE to the reference checkout (tools/idol_packed.py)")
    sys.path.insert(0, str(Path(ref) / "tools"))
    import torch
    from idol_packed import PackedLinear

    q4k = q4_k_cases()
    deq = np.asarray(gguf.dequantize(q4k.reshape(ROWS, -1), gguf.GGMLQuantizationType.Q4_K),
                     dtype=np.float32).reshape(ROWS, COLS)
    src = SimpleNamespace(shape=np.array([COLS, ROWS]), tensor_type=gguf.GGMLQuantizationType.Q4_K, data=q4k)
    ref_deq = PackedLinear(src, None).dequantize(torch.float32).numpy()
    np.savez_compressed(OUT / "q4_k.npz", q4k=q4k, rows=ROWS, cols=COLS, gguf_dequant=deq, ref_dequant=ref_deq)
    print(f"q4_k.npz: {(OUT / 'q4_k.npz').stat().st_size} bytes, rows={ROWS} cols={COLS}")


if __name__ == "__main__":
    main()
