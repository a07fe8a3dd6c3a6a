"""The multi-GPU host logic on CPU: world-size-2 gloo ranks (127.0.0.1), no GPU.

* image_shard covers every image exactly once, contiguously, for any world size;
* the column-parallel linear (all-gather along the features) equals the full linear on every rank, with a torch fp32
  product standing in for the per-rank GPU GEMM;
* max_over_ranks returns the slowest rank's time on every rank.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_image_shard_partitions(pkg):
    from idol_b200.shard import column_range, image_shard
    for images in (0, 1, 7, 64):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                first, count = image_shard(images, r, world)
                seen.extend(range(first, first + count))
            assert seen == list(range(images)), (images, world)
    for n in (14, 480, 1024, 4096, 3072):
        for world in (1, 2, 4, 8):
            cols = []
            for r in range(world):
                first, count = column_range(n, r, world)
                assert first % 128 == 0 or count == 0
                cols.extend(range(first, first + count))
            assert cols == list(range(n)), (n, world)
    with pytest.raises(ValueError):
        image_shard(4, 2, 2)


def _worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import sys
        from pathlib import Path
        sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
        import __graft_entry__
        __graft_entry__.load_package()
        from idol_b200.shard import column_parallel_linear, max_over_ranks
        g = torch.Generator().manual_seed(0)  # same weights and input on every rank
        w = torch.randn((1000, 256), generator=g)
        x = torch.randn((37, 256), generator=g)

        def local(xx, first, count):
            return xx @ w[first:first + count].T

        y = column_parallel_linear(x, 1000, local)
        full = x @ w.T
        slowest = max_over_ranks(1.0 + rank)
        result[rank] = (bool(torch.equal(y, full)), slowest)
    finally:
        dist.destroy_process_group()


def test_column_parallel_and_max_over_ranks_gloo(pkg):
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert result[0] == (True, 2.0) and result[1] == (True, 2.0)
