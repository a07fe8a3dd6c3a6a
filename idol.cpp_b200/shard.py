"""Multi-GPU plumbing of the hot path (scope row (e)): one process per GPU over torch.distributed.

* Request sharding (config 5): independent images are split contiguously across ranks; every rank holds a full
  replica of the Q8_0 weights and runs its images through the stack on its own GPU. There is no collective on the
  data path - `image_shard` is the whole of it.
* Optional column-parallel split (single-image latency): a linear's output features are split across ranks
  (`column_range`); each rank computes its slice with the Q8_0 GEMM over its own rows of W, and the slices are
  all-gathered along the feature dimension. Each rank computes exactly the output columns the single-GPU run computes
  (no partial-sum reduction), so the gathered result equals the 1-GPU result bit for bit.

`column_parallel_linear` takes the per-rank compute as a callable (a CPU stand-in in the gloo tests);
`column_parallel_block_forward_` is the GPU form for one denoiser block, its MLP split this way over NCCL.
"""
from __future__ import annotations

from typing import Callable, Tuple

import torch
import torch.distributed as dist


def image_shard(images: int, rank: int, world: int) -> Tuple[int, int]:
    """(first image, count) of this rank's contiguous share; the first `images % world` ranks take one more."""
    if world < 1 or not 0 <= rank < world or images < 0:
        raise ValueError("image_shard: bad rank/world/images")
    base, extra = divmod(images, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def column_range(n: int, rank: int, world: int, align: int = 128) -> Tuple[int, int]:
    """(first column, count) of this rank's slice of n output features, in multiples of `align` (the GEMM's weight
    tile) except for the last rank, which takes the remainder."""
    if world < 1 or not 0 <= rank < world or n < 1:
        raise ValueError("column_range: bad rank/world/n")
    units = (n + align - 1) // align
    first_u, count_u = image_shard(units, rank, world)
    first = first_u * align
    end = min(n, (first_u + count_u) * align)
    return first, max(0, end - first)


def column_parallel_linear(x: torch.Tensor, n: int, local: Callable[[torch.Tensor, int, int], torch.Tensor],
                           group=None) -> torch.Tensor:
    """y = x . W^T over all n output features, with this rank computing columns column_range(n) by
    local(x, first, count) -> [rows, count], then an all-gather along the features. Every rank returns the full y."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    first, count = column_range(n, rank, world)
    part = local(x, first, count).contiguous()
    rows = x.shape[0]
    counts = [column_range(n, r, world)[1] for r in range(world)]
    width = max(counts)
    padded = part.new_zeros((rows, width))
    padded[:, :count] = part
    gathered = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(gathered, padded, group=group)
    return torch.cat([g[:, :c] for g, c in zip(gathered, counts)], dim=1)


def column_parallel_block_forward_(block, x: torch.Tensor, images: int = 1, group=None, gather_events=None):
    """One DenoiserBlock over a single request with its MLP split across the ranks of `group` (the single-request
    latency option of the multi-GPU plan). Every rank runs the attention half on the whole request (LN -> QKV ->
    rms q,k -> attention -> out + residual: the kernels DenoiserBlock.forward_ launches). ff1 (GELU) and ff2
    (+ residual) then each compute this rank's column_range of their output features with whole-K GEMMs
    (GEMM_WHOLE_K), and an NCCL all-gather along the features rebuilds the full activation on every rank. Each rank
    computes exactly the columns the one-GPU block computes, in the same order, so x afterwards equals
    block.forward_(x) on one GPU bit for bit, on every rank.

    x: [images * tokens, D] fp32, contiguous, on this rank's GPU; updated in place. The feature widths of ff1 and
    ff2 must split evenly over the ranks in multiples of 128 (true for 1024 and 4096 at 2, 4 and 8 ranks).
    gather_events: an optional list that receives a (start, end) pair of timing CUDA events around each all-gather.
    """
    from . import _capi as C
    from . import layers
    qkv_w, out_w, ff1_w, ff2_w = block.weights
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    rows, D = x.shape
    H, heads = ff1_w.out, block.heads
    if x.dtype != torch.float32 or not x.is_contiguous() or D != block.dim or rows % images:
        raise ValueError("column_parallel_block_forward_: x must be a contiguous fp32 [images * tokens, D] tensor")
    for n in (H, D):
        if n % (128 * world):
            raise ValueError("column_parallel_block_forward_: feature widths must split into 128-column slices")
    dev = x.device
    h = torch.empty((rows, D), dtype=torch.bfloat16, device=dev)
    qkv = torch.empty((rows, 3 * D), dtype=torch.bfloat16, device=dev)
    att = torch.empty((rows, D), dtype=torch.bfloat16, device=dev)
    layers.norm_rows(x, block.eps, out=h)
    qkv_w(h, out=qkv)
    layers.rms_heads_(qkv[:, :2 * D], 2 * heads, torch.cat([block.q_gamma, block.k_gamma]))
    layers.attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], heads, batch=images, out=att)
    out_w(att, residual=x, out=x)
    layers.norm_rows(x, block.eps, out=h)

    def gather(part, width):
        full = torch.empty((world,) + tuple(part.shape), dtype=part.dtype, device=dev)
        if gather_events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        dist.all_gather_into_tensor(full, part, group=group)
        if gather_events is not None:
            ev[1].record()
            gather_events.append(ev)
        return full.permute(1, 0, 2).reshape(rows, world * width)

    f0, fw = column_range(H, rank, world)
    part = torch.empty((rows, fw), dtype=torch.bfloat16, device=dev)
    ff1_w(h, act=C.ACT_GELU_TANH, out=part, cols=(f0, fw), flags=C.GEMM_WHOLE_K)
    f1 = gather(part, fw)
    d0, dw = column_range(D, rank, world)
    part2 = torch.empty((rows, dw), dtype=torch.float32, device=dev)
    ff2_w(f1, residual=x[:, d0:], out=part2, cols=(d0, dw), flags=C.GEMM_WHOLE_K)
    x.copy_(gather(part2, dw))
    return x


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The maximum of a per-rank scalar (timings are reported as the max over ranks)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
