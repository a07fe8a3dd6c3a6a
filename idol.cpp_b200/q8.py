"""PyTorch boundary of the Q8_0 linear path: the ``idol_b200::q8_linear`` custom op and drop-in mirrors of the
reference's ``fused_linear`` (tools/idol_triton.py:94-126) and ``PackedLinear`` / ``enable_fused_packed``
(tools/idol_packed.py:12-94).

Weights live on the GPU in the tiled layout the kernels stream (codes int8 + fp16 scales, made once from the GGUF
Q8_0 bytes by the repack kernel). Every call goes to libidol_b200.so through its C-ABI on torch's current stream; if
the library is missing the call raises, it never falls back to another implementation.
"""
from __future__ import annotations

import collections
import ctypes
import weakref
from typing import Optional

import torch
import torch.nn.functional as F

from . import _capi as C

Q8_0_KIND = 8  # tools/idol_triton.py kind code for GGML Q8_0
Q4_0_KIND = 4  # ... and for GGML Q4_0
_GGML_Q8_0 = 8  # gguf.GGMLQuantizationType.Q8_0 enum value
_GGML_Q4_0 = 2  # gguf.GGMLQuantizationType.Q4_0 enum value
Q4_K_KIND = 44  # ... and for GGML Q4_K
_GGML_Q4_K = 12  # gguf.GGMLQuantizationType.Q4_K enum value

_DTYPES = {torch.float32: C.F32, torch.float16: C.F16, torch.bfloat16: C.BF16}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


# ------------------------------------------------------------------------------------------------ format kernels
def q8_bytes(n: int, k: int) -> int:
    return n * (k // 32) * 34


def quantize(w: torch.Tensor) -> torch.Tensor:
    """fp32 CUDA weights [rows, cols] -> Q8_0 bytes [rows * cols / 32 * 34] (uint8), byte-equal to gguf-py 0.19.0."""
    if not w.is_cuda or w.dtype != torch.float32 or w.dim() != 2 or w.shape[1] % 32:
        raise ValueError("quantize: expected a 2-D float32 CUDA tensor with a multiple of 32 columns")
    w = w.contiguous()
    out = torch.empty(w.shape[0] * (w.shape[1] // 32) * 34, dtype=torch.uint8, device=w.device)
    C.check(C.lib().idol_b200_q8_quantize(_ptr(w), w.shape[0], w.shape[1], _ptr(out), _stream(w.device)))
    return out


def tiled_bytes(n: int, k: int) -> int:
    return int(C.lib().idol_b200_q8_tiled_bytes(n, k))


def repack(packed: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """GGUF Q8_0 bytes (CUDA uint8) -> the tiled device layout (uint8): chunks of 128 rows x 64 k, each 8192 code
    bytes followed by their 512 bytes of fp16 scales."""
    if not packed.is_cuda or packed.dtype != torch.uint8 or packed.numel() != q8_bytes(n, k):
        raise ValueError("repack: expected CUDA uint8 Q8_0 bytes of the given shape")
    packed = packed.contiguous()
    tiles = torch.empty(tiled_bytes(n, k), dtype=torch.uint8, device=packed.device)
    C.check(C.lib().idol_b200_q8_repack(_ptr(packed), n, k, _ptr(tiles), _stream(packed.device)))
    return tiles


def q4_0_bytes(n: int, k: int) -> int:
    v = C.lib().idol_b200_q4_0_bytes(n, k)
    if v < 0:
        raise ValueError(f"invalid Q4_0 shape ({n}, {k})")
    return v


def repack_q4_0(packed: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """GGUF Q4_0 bytes (CUDA uint8) -> the tiled device layout. A Q4_0 block is exactly a Q8_0 block with codes
    nibble - 8 (tools/idol_triton.py:48-61), so the result feeds every tiled-layout kernel unchanged."""
    if not packed.is_cuda or packed.dtype != torch.uint8 or packed.numel() != q4_0_bytes(n, k):
        raise ValueError("repack_q4_0: expected CUDA uint8 Q4_0 bytes of the given shape")
    packed = packed.contiguous()
    tiles = torch.empty(tiled_bytes(n, k), dtype=torch.uint8, device=packed.device)
    C.check(C.lib().idol_b200_q4_0_repack(_ptr(packed), n, k, _ptr(tiles), _stream(packed.device)))
    return tiles


def q4_k_bytes(n: int, k: int) -> int:
    v = C.lib().idol_b200_q4_k_bytes(n, k)
    if v < 0:
        raise ValueError(f"invalid Q4_K shape ({n}, {k}): K must be a positive multiple of 256")
    return v


def q4_k_tiled_bytes(n: int, k: int) -> int:
    v = C.lib().idol_b200_q4_k_tiled_bytes(n, k)
    if v < 0:
        raise ValueError(f"invalid Q4_K shape ({n}, {k}): K must be a positive multiple of 256")
    return v


def repack_q4_k(packed: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """GGUF Q4_K bytes (CUDA uint8) -> the Q4_K tiled layout: 4-bit codes plus fp32 A = d sc and B = dmin m per
    32-deep sub-block, from which the kernels form the reference's fp32 weight A code - B exactly
    (tools/idol_packed.py:41-54)."""
    if not packed.is_cuda or packed.dtype != torch.uint8 or packed.numel() != q4_k_bytes(n, k):
        raise ValueError("repack_q4_k: expected CUDA uint8 Q4_K bytes of the given shape")
    packed = packed.contiguous()
    if packed.data_ptr() % 16:
        packed = packed.clone()
    tiles = torch.empty(q4_k_tiled_bytes(n, k), dtype=torch.uint8, device=packed.device)
    C.check(C.lib().idol_b200_q4_k_repack(_ptr(packed), n, k, _ptr(tiles), _stream(packed.device)))
    return tiles


def unpack(tiles: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """Tiled layout -> GGUF Q8_0 bytes, the exact inverse of ``repack``."""
    out = torch.empty(q8_bytes(n, k), dtype=torch.uint8, device=tiles.device)
    C.check(C.lib().idol_b200_q8_unpack(_ptr(tiles), n, k, _ptr(out), _stream(tiles.device)))
    return out


# ------------------------------------------------------------------------------------------------- the custom op
_views: "collections.OrderedDict[tuple, int]" = collections.OrderedDict()
_VIEW_CACHE = 4096


def _tiles_format(tiles, n, k):
    """Q8_0 (also converted Q4_0) or Q4_K tiles, told apart by their size (8704 or 6144 bytes per chunk)."""
    if tiles.numel() == tiled_bytes(n, k):
        return 0
    if k % 256 == 0 and tiles.numel() == q4_k_tiled_bytes(n, k):
        return 1
    raise ValueError(f"tiles of {tiles.numel()} bytes are neither Q8_0 nor Q4_K tiles of shape ({n}, {k})")


def _view(tiles, bias, n, k, device_index):
    """A C-ABI matrix handle over tensors the caller holds (cached; a handle is a few host bytes)."""
    fmt = _tiles_format(tiles, n, k)
    key = (tiles.data_ptr(), 0 if bias is None else bias.data_ptr(), n, k, device_index, fmt)
    h = _views.get(key)
    if h is not None:
        _views.move_to_end(key)
        return h
    out = ctypes.c_void_p()
    make = C.lib().idol_b200_q4_k_view if fmt == 1 else C.lib().idol_b200_q8_view
    C.check(make(_ptr(tiles), _ptr(bias), n, k, device_index, ctypes.byref(out)))
    _views[key] = out.value
    if len(_views) > _VIEW_CACHE:
        _, old = _views.popitem(last=False)
        C.lib().idol_b200_q8_free(ctypes.c_void_p(old))
    return out.value


def gemm_into(y: torch.Tensor, x: torch.Tensor, tiles: torch.Tensor, bias: Optional[torch.Tensor], n: int, k: int,
              n_offset: int = 0, n_count: Optional[int] = None, residual: Optional[torch.Tensor] = None,
              act: int = C.ACT_NONE, flags: int = 0) -> torch.Tensor:
    """y[m, :n_count] = x . W[n_offset:n_offset+n_count]^T + bias (+ residual) (-> act), written into y (2-D, rows of
    any stride >= n_count). x: 2-D bf16/f16 CUDA tensor with unit column stride. residual may alias y."""
    n_count = n - n_offset if n_count is None else n_count
    h = _view(tiles, bias, n, k, x.device.index)
    ldr = 0 if residual is None else residual.stride(0)
    C.check(C.lib().idol_b200_q8_gemm(ctypes.c_void_p(h), _ptr(x), _DTYPES[x.dtype], x.shape[0], x.stride(0),
                                      n_offset, n_count, _ptr(residual), ldr, act, flags, _ptr(y), _DTYPES[y.dtype],
                                      y.stride(0), _stream(x.device)))
    return y


def _aligned_rows(x2: torch.Tensor) -> torch.Tensor:
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    return x2


@torch.library.custom_op("idol_b200::q8_linear", mutates_args=())
def q8_linear(x: torch.Tensor, tiles: torch.Tensor, bias: Optional[torch.Tensor], n: int, k: int, act: int = 0,
              flags: int = 0) -> torch.Tensor:
    """x [..., k] bf16/f16 -> [..., n] in x's dtype; tiles from ``repack`` / ``repack_q4_0`` / ``repack_q4_k``; bias
    is fp32 [n] or None."""
    x2 = _aligned_rows(x.reshape(-1, k))
    y = torch.empty((x2.shape[0], n), dtype=x.dtype, device=x.device)
    if x2.shape[0]:
        gemm_into(y, x2, tiles, bias, n, k, act=act, flags=flags)
    return y.reshape(*x.shape[:-1], n)


@q8_linear.register_fake
def _(x, tiles, bias, n, k, act=0, flags=0):
    return x.new_empty((*x.shape[:-1], n))


# ------------------------------------------------------------------------------------ fused_linear (drop-in)
_tiled_cache: "collections.OrderedDict[tuple, tuple]" = collections.OrderedDict()


def _tiled_for(packed: torch.Tensor, n: int, k: int, kind: int = Q8_0_KIND):
    """The tiled copy of `packed`, made once. An entry is used only while it still belongs to this very tensor (a weak
    reference checked by identity): a freed buffer's address and version are reused by later tensors."""
    key = (packed.data_ptr(), packed.numel(), packed._version, n, k, packed.device.index, kind)
    hit = _tiled_cache.get(key)
    if hit is not None and hit[0]() is packed:
        _tiled_cache.move_to_end(key)
        return hit[1]
    pack = {Q4_0_KIND: repack_q4_0, Q4_K_KIND: repack_q4_k}.get(kind, repack)
    tiles = pack(packed, n, k)
    _tiled_cache[key] = (weakref.ref(packed), tiles)
    if len(_tiled_cache) > 256:
        _tiled_cache.popitem(last=False)
    return tiles


def fused_linear(value, packed, shape, kind, bias=None):
    """Multiply FP16/BF16 activations by Q8_0 (kind 8), Q4_0 (kind 4) or Q4_K (kind 44) weights on CUDA, with the
    contract of tools/idol_triton.py:94-126: same argument checks and ValueError messages, output in value's dtype,
    bias added after the product is rounded to that dtype. Q4_0 runs the Q8_0 kernels (an exact conversion to the
    tiled Q8_0 layout); Q4_K runs them on its own tiled layout, which the kernels dequantise as A code - B."""
    if (not value.is_cuda or not packed.is_cuda or packed.dtype != torch.uint8
            or value.device != packed.device or value.dtype not in (torch.float16, torch.bfloat16)
            or len(shape) != 2 or value.shape[-1] != shape[1] or kind not in (4, 8, 44)):
        raise ValueError('unsupported fused linear input')
    if torch.is_grad_enabled() and (value.requires_grad or (bias is not None and bias.requires_grad)):
        raise ValueError('fused linear supports inference only')
    n, k = shape
    group, size = (256, 144) if kind == 44 else (32, 18 if kind == 4 else 34)
    if n < 1 or k < 1 or k % group or packed.numel() != n * (k // group) * size:
        raise ValueError('invalid packed linear dimensions')
    if bias is not None and (bias.shape != (n,) or bias.device != value.device or bias.dtype != value.dtype):
        raise ValueError('invalid fused linear bias')
    tiles = _tiled_for(packed, n, k, kind)
    b32 = None if bias is None else bias.float()
    return torch.ops.idol_b200.q8_linear(value, tiles, b32, n, k, C.ACT_NONE, C.EPI_BIAS_AFTER_ROUND)


# ----------------------------------------------------------------------------------- PackedLinear (drop-in)
class PackedLinear(torch.nn.Module):
    """Mirror of tools/idol_packed.py:12-82 for Q8_0, Q4_0 and Q4_K matrices (the kinds the reference's fused path
    takes): keeps the GGUF bytes as the ``packed`` buffer, and when ``fused`` is set and the input is CUDA fp16/bf16
    without grad, runs the sm_100a kernels on a tiled copy made once per device. Unfused calls expand the weights (our
    dequant kernels on CUDA) and use F.linear, as the reference's expansion path does. The reference's expansion-only
    kinds (F16, Q2_K, Q6_K) are outside this build and raise ValueError here."""

    def __init__(self, source, bias):
        super().__init__()
        self.shape = tuple(reversed([int(s) for s in source.shape]))
        self.kind = int(source.tensor_type)
        if len(self.shape) != 2 or self.kind not in (_GGML_Q8_0, _GGML_Q4_0, _GGML_Q4_K):
            raise ValueError("unsupported packed matrix")
        import numpy as np
        self.register_buffer("packed", torch.from_numpy(np.array(source.data, copy=True)).reshape(-1))
        self.bias = torch.nn.Parameter(bias.detach(), requires_grad=False) if bias is not None else None
        self.fused = False
        self._tiled = None

    def _tiles(self):
        # Valid while it was made from this very buffer at this version (moving the module replaces the buffer).
        if (self._tiled is None or self._tiled[0]() is not self.packed
                or self._tiled[1] != self.packed._version):
            pack = {_GGML_Q4_0: repack_q4_0, _GGML_Q4_K: repack_q4_k}.get(self.kind, repack)
            self._tiled = (weakref.ref(self.packed), self.packed._version, pack(self.packed, *self.shape))
        return self._tiled[2]

    def dequantize(self, dtype):
        n, k = self.shape
        if self.packed.is_cuda:
            return dequantize_tiled(self._tiles(), n, k, dtype)
        if self.kind == _GGML_Q4_K:  # 144-byte super-blocks of 256: d, dmin, 6-bit scales / mins, 4-bit codes
            blocks = self.packed.reshape(-1, 144)
            d = blocks[:, :2].contiguous().view(torch.float16).float()
            dmin = blocks[:, 2:4].contiguous().view(torch.float16).float()
            sm = blocks[:, 4:16].reshape(-1, 3, 4)
            lo, mid, top = sm[:, 0], sm[:, 1], sm[:, 2]
            sc = torch.cat((lo & 63, (top & 15) | ((lo >> 2) & 48)), dim=1).float()
            mn = torch.cat((mid & 63, (top >> 4) | ((mid >> 2) & 48)), dim=1).float()
            q = blocks[:, 16:].reshape(-1, 4, 1, 32)
            codes = torch.cat(((q & 15), (q >> 4)), dim=2).reshape(-1, 8, 32).float()
            w = (d * sc).reshape(-1, 8, 1) * codes - (dmin * mn).reshape(-1, 8, 1)
            return w.reshape(self.shape).to(dtype)
        if self.kind == _GGML_Q4_0:  # 18-byte blocks: fp16 d, then low nibbles = elements 0-15, high = 16-31
            blocks = self.packed.reshape(-1, 18)
            nib = blocks[:, 2:]
            codes = (torch.cat((nib & 15, nib >> 4), dim=1).to(torch.int16) - 8).float()
        else:
            blocks = self.packed.reshape(-1, 34)
            codes = blocks[:, 2:].contiguous().view(torch.int8).float()
        scale = blocks[:, :2].contiguous().view(torch.float16).float()
        return (codes * scale).reshape(self.shape).to(dtype)

    def forward(self, value):
        needs_grad = torch.is_grad_enabled() and (value.requires_grad or
                                                  (self.bias is not None and self.bias.requires_grad))
        if self.fused and value.is_cuda and value.dtype in (torch.float16, torch.bfloat16) and not needs_grad:
            kind = {_GGML_Q4_0: Q4_0_KIND, _GGML_Q4_K: Q4_K_KIND}.get(self.kind, Q8_0_KIND)
            return fused_linear(value, self.packed, self.shape, kind, self.bias)
        return F.linear(value, self.dequantize(value.dtype), self.bias)


def enable_fused_packed(model):
    """Enable supported packed layers; return the number configured (tools/idol_packed.py:85-94)."""
    count = 0
    for layer in model.modules():
        if isinstance(layer, PackedLinear):
            layer.fused = True
            count += 1
    return count


def dequantize_tiled(tiles, n, k, dtype=torch.float32):
    """Dense [n, k] weights from Q8_0 tiles (d q) or Q4_K tiles (A code - B): fp32 exact, bf16/fp16 rounded from the
    fp32 value."""
    out = torch.empty((n, k), dtype=dtype, device=tiles.device)
    fn = C.lib().idol_b200_q4_k_dequantize if _tiles_format(tiles, n, k) == 1 else C.lib().idol_b200_q8_dequantize
    C.check(fn(_ptr(tiles), n, k, _ptr(out), _DTYPES[out.dtype], _stream(tiles.device)))
    return out
