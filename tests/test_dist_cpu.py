"""Data-parallel host logic on CPU: world-size-2 gloo ranks shard a batch and reduce device times (max over ranks),
as bench.py does across GPUs."""
import os

import pytest


def test_shard_bounds_cover_batch_once():
    from xtagger_b200.dist import shard_bounds
    for batch in (1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            if world > batch:
                continue
            seen = []
            for r in range(world):
                lo, hi = shard_bounds(batch, world, r)
                assert hi - lo in (batch // world, batch // world + 1)
                seen += list(range(lo, hi))
            assert seen == list(range(batch))


def _rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from xtagger_b200.dist import allmax, shard_bounds
    lo, hi = shard_bounds(64, world, rank)
    t = allmax(1.5 + rank)            # rank 1 is the slowest
    dist.barrier()
    q.put((rank, lo, hi, t))
    dist.destroy_process_group()


def test_gloo_two_ranks_shard_and_max():
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert [(lo, hi) for _, lo, hi, _ in res] == [(0, 32), (32, 64)]
    assert all(t == 2.5 for *_, t in res)
