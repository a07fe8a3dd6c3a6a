"""Resident weights and the layer compositions of the hot path, over the C-ABI of libidol_b200.so.

* ``Q8Weight``     - one Q8_0 matrix (+ fp32 bias) resident on a GPU in the tiled layout (idol_b200_q8_import),
                     made once from GGUF Q8_0 bytes, as src/weights.cpp + quantized_linear make theirs once.
* ``DenoiserBlock`` - scope row A14: LN -> QKV -> rms q,k -> attention -> out + res -> LN -> ff1 (GELU tanh) -> ff2 +
                     res (src/decoders.cpp:296-313 without the cross-attention), in place on the residual stream.
* ``GaussianBlock`` - the Gaussian decoder's block (src/decoders.cpp:296-313): the same plus a cross-attention to
                     the latent tokens between the self-attention and the MLP.
* ``DenoiserStack`` - config 5: a stack of DenoiserBlocks run over many independent images, a chunk of images at
                     a time through every block, with one workspace shared by the blocks.
* ``GaussianMLP``  - scope row A15: 128 -> 512 (SiLU) -> 512 (SiLU) -> 14 -> activated heads.

Workspaces are device tensors owned by the Python objects and reused across calls.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _capi as C
from .q8 import _DTYPES, _ptr, _stream, q8_bytes, quantize


class Q8Weight:
    """A resident Q8_0 matrix. `q8` is GGUF Q8_0 bytes (uint8, out*in/32*34) on the target CUDA device."""

    def __init__(self, q8: torch.Tensor, out: int, inp: int, bias: Optional[torch.Tensor] = None):
        if not q8.is_cuda or q8.dtype != torch.uint8 or q8.numel() != q8_bytes(out, inp):
            raise ValueError("Q8Weight: expected CUDA uint8 Q8_0 bytes of the given shape")
        self.out, self.inp, self.device = out, inp, q8.device
        b = None if bias is None else bias.detach().to(device=q8.device, dtype=torch.float32).contiguous()
        h = ctypes.c_void_p()
        C.check(C.lib().idol_b200_q8_import(_ptr(q8.contiguous()), q8.numel(), out, inp, _ptr(b), q8.device.index,
                                            _stream(q8.device), ctypes.byref(h)))
        torch.cuda.current_stream(q8.device).synchronize()
        self.handle = h.value
        self.q8 = q8

    @classmethod
    def from_float(cls, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> "Q8Weight":
        """Quantize fp32 CUDA weights [out, in] on the device (gguf-py Q8_0 semantics) and upload."""
        return cls(quantize(w.float().contiguous()), w.shape[0], w.shape[1], bias)

    def __call__(self, x: torch.Tensor, act: int = C.ACT_NONE, residual: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                 cols: Optional[tuple] = None, flags: int = 0) -> torch.Tensor:
        """y = x W^T + b (+ residual) (-> act). `cols` = (first, count) computes only output features first ..
        first + count - 1 (src/kernels.hpp:75-76 gemm_packed's window): `out` and `residual` then hold just those
        columns. `flags`: IDOL_* GEMM flags (C.GEMM_WHOLE_K keeps a window equal to the full product bit for bit)."""
        x2 = x if (x.stride(-1) == 1 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0) else x.contiguous()
        first, count = (0, self.out) if cols is None else (int(cols[0]), int(cols[1]))
        if out is None:
            out = torch.empty((x2.shape[0], count), dtype=out_dtype or x.dtype, device=x.device)
        if out.dim() != 2 or out.stride(1) != 1 or out.shape[1] < count or out.shape[0] != x2.shape[0]:
            raise ValueError("Q8Weight: out must be a [rows, >= count] tensor with unit column stride")
        ldr = 0 if residual is None else residual.stride(0)
        C.check(C.lib().idol_b200_q8_gemm(ctypes.c_void_p(self.handle), _ptr(x2), _DTYPES[x2.dtype], x2.shape[0],
                                          x2.stride(0), first, count, _ptr(residual), ldr, act, flags, _ptr(out),
                                          _DTYPES[out.dtype], out.stride(0), _stream(x.device)))
        return out

    def heads(self, x: torch.Tensor, head_cols: int, head_split: int, gamma_a: torch.Tensor,
              gamma_b: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """bf16 y = x W^T + b, then rms_heads of columns [0, head_split) with gamma_a and [head_split, head_cols) with
        gamma_b (src/decoders.cpp:234-237, 298-300), the norm fused into the GEMM's epilogue where it can be."""
        x2 = x if (x.stride(-1) == 1 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0) else x.contiguous()
        if x2.dtype != torch.bfloat16:
            raise ValueError("Q8Weight.heads: x must be bf16")
        if out is None:
            out = torch.empty((x2.shape[0], self.out), dtype=torch.bfloat16, device=x.device)
        ga = gamma_a.detach().to(device=x.device, dtype=torch.float32).contiguous()
        gb = None if gamma_b is None else gamma_b.detach().to(device=x.device, dtype=torch.float32).contiguous()
        C.check(C.lib().idol_b200_q8_gemm_heads(ctypes.c_void_p(self.handle), _ptr(x2), x2.shape[0], x2.stride(0),
                                                _ptr(out), out.stride(0), head_cols, head_split, _ptr(ga), _ptr(gb),
                                                _stream(x.device)))
        return out

    def int8act(self, x: torch.Tensor, act: int = C.ACT_NONE, residual: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32,
                cols: Optional[tuple] = None) -> torch.Tensor:
        """The same linear on integer activations, the reference's set_quant_kernel(1) path (src/kernels.cpp:368-479):
        x (fp32, bf16 or f16) is quantized per (row, 32-group) to int8 and the groups' integer dot products are
        scaled and summed in the reference's order, so the result equals that kernel's bit for bit."""
        if x.dim() != 2 or x.stride(1) != 1 or x.dtype not in _DTYPES:
            raise ValueError("Q8Weight.int8act: x must be a 2-D tensor with unit column stride")
        first, count = (0, self.out) if cols is None else (int(cols[0]), int(cols[1]))
        if out is None:
            out = torch.empty((x.shape[0], count), dtype=out_dtype, device=x.device)
        nbytes = int(C.lib().idol_b200_q8_gemm_int8act_workspace_bytes(x.shape[0], self.inp))
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
        ldr = 0 if residual is None else residual.stride(0)
        C.check(C.lib().idol_b200_q8_gemm_int8act(ctypes.c_void_p(self.handle), _ptr(x), _DTYPES[x.dtype], x.shape[0],
                                                  x.stride(0), first, count, _ptr(residual), ldr, act, _ptr(out),
                                                  _DTYPES[out.dtype], out.stride(0), _ptr(ws), ws.numel(),
                                                  _stream(x.device)))
        return out

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            try:
                C.lib().idol_b200_q8_free(ctypes.c_void_p(h))
            except Exception:
                pass
            self.handle = None


class _Workspace:
    def __init__(self):
        self.buf = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        return self.buf


class DenoiserBlock:
    """Scope row A14 on resident Q8_0 weights. `layers` maps qkv/out/ff1/ff2 to Q8Weight; gammas are [D] tensors."""

    def __init__(self, qkv: Q8Weight, out: Q8Weight, ff1: Q8Weight, ff2: Q8Weight, q_gamma: torch.Tensor,
                 k_gamma: torch.Tensor, heads: int, eps: float = 1e-6):
        self.weights = (qkv, out, ff1, ff2)
        dev = qkv.device
        self.q_gamma = q_gamma.detach().to(device=dev, dtype=torch.float32).contiguous()
        self.k_gamma = k_gamma.detach().to(device=dev, dtype=torch.float32).contiguous()
        h = ctypes.c_void_p()
        C.check(C.lib().idol_b200_block_create(*(ctypes.c_void_p(w.handle) for w in self.weights), _ptr(self.q_gamma),
                                               _ptr(self.k_gamma), heads, float(eps), ctypes.byref(h)))
        self.handle = h.value
        self.dim, self.heads, self.device, self.eps = out.out, heads, dev, float(eps)
        self.ws = _Workspace()

    def workspace_bytes(self, rows: int) -> int:
        return int(C.lib().idol_b200_block_workspace_bytes(ctypes.c_void_p(self.handle), rows))

    def forward_(self, x: torch.Tensor, images: int = 1) -> torch.Tensor:
        """In place on x: [images * tokens, D], fp32 or bf16, contiguous."""
        if not x.is_contiguous() or x.dim() != 2 or x.shape[1] != self.dim or x.shape[0] % images:
            raise ValueError("DenoiserBlock: x must be a contiguous [images * tokens, D] tensor")
        rows = x.shape[0]
        nbytes = self.workspace_bytes(rows)
        ws = self.ws.get(nbytes, x.device)
        C.check(C.lib().idol_b200_block_forward(ctypes.c_void_p(self.handle), _ptr(x), _DTYPES[x.dtype],
                                                rows // images, images, _ptr(ws), ws.numel(), _stream(x.device)))
        return x

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            try:
                C.lib().idol_b200_block_free(ctypes.c_void_p(h))
            except Exception:
                pass
            self.handle = None


class DenoiserStack:
    """A stack of DenoiserBlocks (the denoiser's 24 transformer blocks, tools/export_full_gguf.py:311-314) over a
    batch of independent sequences: each image's CFG branches are separate sequences of `tokens` rows that attend only
    within themselves (batched CFG, tools/idol_generate.py:153,193). forward_ runs `chunk` sequences at a time through
    every block (so the workspace is sized by the chunk, not the batch). With more than one chunk, consecutive chunks
    go to `lanes` CUDA streams in turn (the caller's current stream and side streams the stack owns), each with its own
    workspace: the chunks are independent, and the small memory-bound launches of one (LayerNorms, the GEMMs' weight
    dequantisation) then run on SMs beside the other's attention or GEMM CTAs. Each chunk's kernels and their order are
    the same in every lane count, so the result does not depend on it."""

    def __init__(self, blocks: Sequence[DenoiserBlock]):
        if not blocks:
            raise ValueError("DenoiserStack: no blocks")
        self.blocks = tuple(blocks)
        self.dim, self.device = self.blocks[0].dim, self.blocks[0].device
        if any(b.dim != self.dim or b.device != self.device for b in self.blocks):
            raise ValueError("DenoiserStack: blocks of different widths or devices")
        self._ws = {}          # CUDA stream handle -> _Workspace (calls on different streams never share one)
        self._side = []        # side streams of the lanes

    def _workspace(self, stream: "torch.cuda.Stream", nbytes: int, device) -> torch.Tensor:
        # Allocated in the lane's stream order, so that the caching allocator hands the memory out again only in that
        # order once the buffer is replaced.
        with torch.cuda.stream(stream):
            return self._ws.setdefault(stream.cuda_stream, _Workspace()).get(nbytes, device)

    def forward_(self, x: torch.Tensor, sequences: int, chunk: Optional[int] = None, lanes: int = 2) -> torch.Tensor:
        """In place on x: [sequences * tokens, D] (fp32 or bf16, contiguous), `chunk` sequences per pass through the
        blocks (all of them by default). Launches on the current stream, which waits for the side lanes before this
        call returns (in stream order: nothing synchronises with the host)."""
        if not x.is_contiguous() or x.dim() != 2 or x.shape[1] != self.dim or sequences < 1 or x.shape[0] % sequences:
            raise ValueError("DenoiserStack: x must be a contiguous [sequences * tokens, D] tensor")
        tokens = x.shape[0] // sequences
        chunk = sequences if chunk is None else max(1, min(int(chunk), sequences))
        starts = list(range(0, sequences, chunk))
        lanes = max(1, min(int(lanes), len(starts)))
        lib = C.lib()
        main = torch.cuda.current_stream(x.device)
        while len(self._side) < lanes - 1:
            self._side.append(torch.cuda.Stream(device=x.device))
        streams = [main] + self._side[:lanes - 1]
        nbytes = self.blocks[0].workspace_bytes(chunk * tokens)
        ws = [self._workspace(st, nbytes, x.device) for st in streams]
        for st in streams[1:]:
            st.wait_stream(main)  # x and the workspaces were last touched in the main stream's order
        for i, s0 in enumerate(starts):
            lane = i % lanes
            n = min(chunk, sequences - s0)
            part = x[s0 * tokens:(s0 + n) * tokens]
            for b in self.blocks:
                C.check(lib.idol_b200_block_forward(ctypes.c_void_p(b.handle), _ptr(part), _DTYPES[x.dtype], tokens,
                                                    n, _ptr(ws[lane]), ws[lane].numel(), streams[lane].cuda_stream))
        for st in streams[1:]:
            main.wait_stream(st)
        return x


class GaussianBlock:
    """The Gaussian decoder's block (src/decoders.cpp:296-313): DenoiserBlock's sublayers plus the cross-attention to
    the latent tokens. Weights: Q8Weight for qkv/out/cross_q/cross_out/ff1/ff2; fp32 tensors for the gammas, norm2's
    gamma/beta ([D]) and the dense to_kv weight [2D, cond_dim] and bias [2D]."""

    def __init__(self, qkv: Q8Weight, out: Q8Weight, cross_q: Q8Weight, cross_out: Q8Weight, ff1: Q8Weight,
                 ff2: Q8Weight, q_gamma, k_gamma, cross_q_gamma, cross_k_gamma, norm2_gamma, norm2_beta,
                 kv_weight: torch.Tensor, kv_bias: Optional[torch.Tensor], heads: int, eps: float = 1e-6):
        self.weights = (qkv, out, cross_q, cross_out, ff1, ff2)
        dev = qkv.device

        def f32(t):
            return t.detach().to(device=dev, dtype=torch.float32).contiguous()

        self.vectors = [f32(t) for t in (q_gamma, k_gamma, cross_q_gamma, cross_k_gamma, norm2_gamma, norm2_beta)]
        self.kv_weight = f32(kv_weight)
        self.kv_bias = None if kv_bias is None else f32(kv_bias)
        self.cond_dim = self.kv_weight.shape[1]
        h = ctypes.c_void_p()
        C.check(C.lib().idol_b200_gs_block_create(*(ctypes.c_void_p(w.handle) for w in self.weights),
                                                  *(_ptr(v) for v in self.vectors), _ptr(self.kv_weight),
                                                  _ptr(self.kv_bias), self.cond_dim, heads, float(eps),
                                                  ctypes.byref(h)))
        self.handle = h.value
        self.dim, self.heads, self.device = out.out, heads, dev
        self.ws = _Workspace()

    def workspace_bytes(self, rows: int, cond_rows_total: int) -> int:
        return int(C.lib().idol_b200_gs_block_workspace_bytes(ctypes.c_void_p(self.handle), rows, cond_rows_total))

    def forward_(self, x: torch.Tensor, cond: torch.Tensor, images: int = 1) -> torch.Tensor:
        """In place on x: [images * tokens, D] (fp32 or bf16, contiguous); cond: fp32 [images * cond_rows,
        cond_dim] on the same device."""
        if not x.is_contiguous() or x.dim() != 2 or x.shape[1] != self.dim or x.shape[0] % images:
            raise ValueError("GaussianBlock: x must be a contiguous [images * tokens, D] tensor")
        if (cond.dtype != torch.float32 or not cond.is_contiguous() or cond.dim() != 2
                or cond.shape[1] != self.cond_dim or cond.shape[0] % images or cond.device != x.device):
            raise ValueError("GaussianBlock: cond must be a contiguous fp32 [images * cond_rows, cond_dim] tensor")
        rows, crows = x.shape[0], cond.shape[0]
        ws = self.ws.get(self.workspace_bytes(rows, crows), x.device)
        C.check(C.lib().idol_b200_gs_block_forward(ctypes.c_void_p(self.handle), _ptr(x), _DTYPES[x.dtype],
                                                   rows // images, images, _ptr(cond), crows // images, _ptr(ws),
                                                   ws.numel(), _stream(x.device)))
        return x

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            try:
                C.lib().idol_b200_gs_block_free(ctypes.c_void_p(h))
            except Exception:
                pass
            self.handle = None


class GaussianMLP:
    """Scope row A15 on resident Q8_0 weights: returns (raw [P, 14] fp32, activated [P, 14] fp32)."""

    def __init__(self, layers: Sequence[Q8Weight]):
        self.layers = tuple(layers)
        h = ctypes.c_void_p()
        C.check(C.lib().idol_b200_gaussian_mlp_create(*(ctypes.c_void_p(w.handle) for w in self.layers),
                                                      ctypes.byref(h)))
        self.handle = h.value
        self.ws = _Workspace()

    def __call__(self, x: torch.Tensor, raw: bool = True):
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
            raise ValueError("GaussianMLP: x must be a 2-D bf16 tensor with unit column stride")
        points = x.shape[0]
        nbytes = int(C.lib().idol_b200_gaussian_mlp_workspace_bytes(ctypes.c_void_p(self.handle), points))
        ws = self.ws.get(nbytes, x.device)
        out = torch.empty((points, 14), dtype=torch.float32, device=x.device)
        raw_t = torch.empty((points, 14), dtype=torch.float32, device=x.device) if raw else None
        C.check(C.lib().idol_b200_gaussian_mlp_forward(ctypes.c_void_p(self.handle), _ptr(x), points, x.stride(0),
                                                       _ptr(ws), ws.numel(), _ptr(raw_t), _ptr(out),
                                                       _stream(x.device)))
        return raw_t, out

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            try:
                C.lib().idol_b200_gaussian_mlp_free(ctypes.c_void_p(h))
            except Exception:
                pass
            self.handle = None
