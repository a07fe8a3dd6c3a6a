"""Writes tests/golden/q4_0.npz, the GGUF Q4_0 (kind 4) golden vectors, from gguf-py 0.19.0 and the reference itself.

Run in a checkout where gguf-py is importable and the reference checkout is given by IDOL_REFERENCE:

    IDOL_REFERENCE=<reference checkout> python tests/golden/make_golden_q4_0.py

q4_0.npz holds fp32 weights (the seeded and edge-case rows of q8_quant.npz's generator), the bytes
gguf.quantize(W, Q4_0) returns for them, gguf.dequantize of those bytes, and the reference's own expansion of them
(tools/idol_packed.py PackedLinear.dequantize, the path its unfused layers take).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "tests" / "golden"))

import gguf  # noqa: E402

from make_golden import quant_cases  # noqa: E402

OUT = Path(__file__).resolve().parent


def main():
    ref = os.environ.get("IDOL_REFERENCE")
    if not ref or not (Path(ref) / "tools" / "idol_packed.py").exists():
        raise SystemExit("set IDOL_REFERENCE to the reference checkout (tools/idol_packed.py)")
    sys.path.insert(0, str(Path(ref) / "tools"))
    import torch
    from idol_packed import PackedLinear

    w, _ = quant_cases()
    rows, cols = w.shape
    q4 = np.asarray(gguf.quantize(np.ascontiguousarray(w, np.float32), gguf.GGMLQuantizationType.Q4_0),
                    dtype=np.uint8)
    deq = np.asarray(gguf.dequantize(q4, gguf.GGMLQuantizationType.Q4_0), dtype=np.float32).reshape(rows, cols)
    # PackedLinear reads shape (reversed), tensor_type and data from a GGUF reader tensor.
    src = SimpleNamespace(shape=np.array([cols, rows]), tensor_type=gguf.GGMLQuantizationType.Q4_0, data=q4)
    ref_deq = PackedLinear(src, None).dequantize(torch.float32).numpy()
    np.savez_compressed(OUT / "q4_0.npz", w=w, q4=q4.reshape(-1), gguf_dequant=deq, ref_dequant=ref_deq)
    print(f"q4_0.npz: {(OUT / 'q4_0.npz').stat().st_size} bytes, rows={rows} cols={cols}")


if __name__ == "__main__":
    main()
