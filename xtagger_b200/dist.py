"""Host-side data parallelism across processes (one per GPU): contiguous shards of the image batch and the
max-over-ranks of device times. There is no collective on the forward itself; torch.distributed only carries the
barrier and the timing reduction."""


def shard_bounds(batch, world, rank):
    """[lo, hi) of the images rank `rank` runs: contiguous shards whose sizes differ by at most one (the same rule
    as the engine's multi-device split)."""
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def allmax(value, group=None):
    """Max of a float over the ranks of the default process group (value itself without one)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
