"""Norms and attention between the Q8_0 linears, on the sm_100a kernels of libidol_b200.so.

Mirrors of the decoders' helpers (src/decoders.cpp:23-42 norm_rows, :74-86 rms_heads) and of
src/kernels.cpp:737-746 attention, taking CUDA tensors (2-D views with unit column stride are accepted as they are,
so q/k/v can be column slices of one packed projection, as the decoders pass them).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _capi as C
from .q8 import _DTYPES, _ptr, _stream


def _f32(t: Optional[torch.Tensor]):
    if t is None:
        return None
    return t.detach().to(dtype=torch.float32).contiguous()


def norm_rows(x: torch.Tensor, eps: float, gamma=None, beta=None, shift=None, scale=None,
              out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """LayerNorm over the last dim of a 2-D CUDA tensor (rows any stride, unit column stride), with optional affine
    gamma/beta and adaLN (1 + scale), shift. `out` may be `x` (in place)."""
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("norm_rows: expected a 2-D tensor with unit column stride")
    rows, dim = x.shape
    if out is None:
        out = torch.empty((rows, dim), dtype=out_dtype or x.dtype, device=x.device)
    g, b, sh, sc = _f32(gamma), _f32(beta), _f32(shift), _f32(scale)
    C.check(C.lib().idol_b200_norm_rows(_ptr(x), _DTYPES[x.dtype], rows, dim, x.stride(0), float(eps), _ptr(g),
                                        _ptr(b), _ptr(sh), _ptr(sc), _ptr(out), _DTYPES[out.dtype], out.stride(0),
                                        _stream(x.device)))
    return out


def rms_heads_(x: torch.Tensor, heads: int, gamma: torch.Tensor, head_dim: int = 64) -> torch.Tensor:
    """In place per-head L2 norm of a 2-D view (e.g. qkv[:, :D]): x * sqrt(hd) / max(|x|, 1e-12) * gamma."""
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("rms_heads_: expected a 2-D view with unit column stride")
    g = _f32(gamma)
    C.check(C.lib().idol_b200_rms_heads(_ptr(x), _DTYPES[x.dtype], x.shape[0], x.stride(0), heads, head_dim, _ptr(g),
                                        _stream(x.device)))
    return x


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, batch: int = 1,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(q k^T / sqrt(64)) v per head for `batch` independent sequences stacked along the rows.
    q: [batch * lq, >= heads*64] bf16 view; k, v: [batch * lk, >= heads*64] views; returns [batch * lq, heads*64] in
    bf16, or in fp32 when `out` is an fp32 tensor."""
    for t in (q, k, v):
        if t.dim() != 2 or t.stride(1) != 1 or t.dtype != torch.bfloat16:
            raise ValueError("attention: expected 2-D bf16 views with unit column stride")
    if k.stride(0) != v.stride(0) or k.shape != v.shape:
        raise ValueError("attention: k and v must have the same shape and row stride")
    dim = heads * 64
    if q.shape[0] % batch or k.shape[0] % batch:
        raise ValueError("attention: rows must split evenly into the batch")
    lq, lk = q.shape[0] // batch, k.shape[0] // batch
    if out is None:
        out = torch.empty((q.shape[0], dim), dtype=torch.bfloat16, device=q.device)
    if out.dtype not in (torch.bfloat16, torch.float32) or out.dim() != 2 or out.stride(1) != 1:
        raise ValueError("attention: out must be a 2-D bf16 or fp32 tensor with unit column stride")
    C.check(C.lib().idol_b200_attention(_ptr(q), lq, q.stride(0), _ptr(k), _ptr(v), lk, k.stride(0), heads, 64,
                                        _ptr(out), _DTYPES[out.dtype], out.stride(0), batch, _stream(q.device)))
    return out
