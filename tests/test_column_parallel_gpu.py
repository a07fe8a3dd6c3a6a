"""The column-parallel denoiser block on two GPUs over NCCL (shard.column_parallel_block_forward_): ff1 and ff2 split by
output features with whole-K GEMM windows, each slice all-gathered. Every rank must end with exactly the one-GPU result,
bit for bit: the same function on a one-rank group (one GPU, full-width whole-K GEMMs) for every size, and
DenoiserBlock.forward_ itself for a request of one image (2 x 4096 tokens), where the one-GPU GEMMs do not split K
either. Needs two CUDA devices; skipped otherwise. The ranks are child processes (spawned, NCCL over 127.0.0.1, a
short process-group timeout)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make_block(dev, seed=11):
    from idol_b200.block import DenoiserBlock, Q8Weight
    g = torch.Generator(device=dev).manual_seed(seed)
    D, H = 1024, 4096
    w = {name: Q8Weight.from_float(torch.randn((n, k), device=dev, generator=g) * 0.02,
                                   torch.randn(n, device=dev, generator=g) * 0.01)
         for name, (n, k) in {"qkv": (3 * D, D), "out": (D, D), "ff1": (H, D), "ff2": (D, H)}.items()}
    return DenoiserBlock(w["qkv"], w["out"], w["ff1"], w["ff2"], 1 + 0.1 * torch.randn(D, device=dev, generator=g),
                         1 + 0.1 * torch.randn(D, device=dev, generator=g), 16)


def _rank(rank, world, port, tokens, images, result):
    import datetime
    import sys

    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import __graft_entry__
    __graft_entry__.load_package()
    from idol_b200.shard import column_parallel_block_forward_
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        solo = [dist.new_group([r]) for r in range(world)]  # every rank creates every group, in the same order
        blk = _make_block(dev)
        g = torch.Generator(device=dev).manual_seed(5)
        x0 = torch.randn((images * tokens, 1024), device=dev, generator=g)
        x = x0.clone()
        for _ in range(2):  # two blocks in a row: the second starts from the gathered result
            column_parallel_block_forward_(blk, x, images=images)
        one = x0.clone()
        for _ in range(2):
            column_parallel_block_forward_(blk, one, images=images, group=solo[rank])
        ref = x0.clone()
        for _ in range(2):
            blk.forward_(ref, images=images)
        torch.cuda.synchronize()
        same = torch.tensor([int(torch.equal(x, one)), int(torch.equal(x, ref))], device=dev)
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        if rank == 0:
            result.put((int(same[0].item()), int(same[1].item()), float((x - one).abs().max()),
                        float((x - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens,images", [(4096, 2), (640, 3)])
def test_column_parallel_block_equals_one_gpu_bit_for_bit(pkg, tokens, images):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, tokens, images, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    same_one, same_block, d_one, d_block = result.get(timeout=5)
    assert same_one == 1, f"column-parallel block differs from its one-GPU whole-K form (max abs diff {d_one})"
    if tokens * images == 8192:
        assert same_block == 1, f"column-parallel block differs from DenoiserBlock.forward_ (max abs diff {d_block})"
