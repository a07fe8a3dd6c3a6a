"""Multi-GPU plumbing of the hot path (scope row (e)): one process per GPU over torch.distributed.

* Request sharding (config 5): independent images are split contiguously across ranks; every rank holds a full
  replica of the Q8_0 weights and runs its images through the stack on its own GPU. There is no collective on the
  data path - `image_shard` is the whole of it.
* Optional column-parallel split (single-image latency): a linear's output features are split across ranks
  (`column_range`); each rank computes its slice with the Q8_0 GEMM over its own rows of W, and the slices are
  all-gathered along the feature dimension. Each rank computes exactly the output columns the single-GPU run computes
  (no partial-sum reduction), so the gathered result equals the 1-GPU result bit for bit.

Nothing here computes; the per-rank compute is a callable (the GPU GEMM in production, a CPU stand-in in the gloo
tests).
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


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The maximum of a per-rank scalar (timings are reported as the max over ranks)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
