"""Data-parallel replicas of the DiT over the GPUs of one node.

Independent pictures (64 generations, distinct seeds) are
split into contiguous shards, one process per GPU, each with its own
libexn_b200 handle on its own device.  Pictures never interact, so there is
no collective on the data path; torch.distributed (NCCL on GPUs, gloo in the
CPU tests) carries only the launch barrier and the max-over-ranks timing.
The reference has no multi-GPU path at all (it serialises requests on one
GPU, src/server.lisp:24-28).
"""
from __future__ import annotations

import os


def shard(n_items: int, rank: int, world: int) -> range:
    """Rank RANK's contiguous share of N_ITEMS (sizes differ by at most 1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank %d of %d" % (rank, world))
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def batches(items: range, batch: int):
    """ITEMS in consecutive batches of at most BATCH."""
    for i in range(items.start, items.stop, batch):
        yield range(i, min(i + batch, items.stop))


def env_rank():
    """(rank, world, local_rank) from the torchrun environment, (0, 1, 0) without one."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def max_over_ranks(dist, value: float, device=None) -> float:
    """The largest VALUE over the ranks of the default group (DIST = torch.distributed or None)."""
    if dist is None or not dist.is_initialized():
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
