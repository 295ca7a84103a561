"""Request sharding across the GPUs of one box: one process per GPU, no collective on the data path.

Every input's result depends only on that input (the reference's llm.py:7-9), so a batch of requests is split into
contiguous shards, each rank runs its shard through its own decoder batch, and the results are gathered back in
request order. The only collectives are host-side: a start barrier, the max of the per-rank device times, and the
ordered gather of results. These helpers work with any ``torch.distributed`` backend (``nccl`` on the GPUs,
``gloo`` on the CPU in the tests).
"""

from __future__ import annotations

from typing import Any, Sequence


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous shard of ``total`` items: the first ``total % world`` ranks take one
    item more, so shard sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if total < 0:
        raise ValueError(f"total {total}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(items: Sequence[Any], world: int, rank: int) -> Sequence[Any]:
    """Rank's contiguous shard of ``items`` (see :func:`shard_bounds`)."""
    a, b = shard_bounds(len(items), world, rank)
    return items[a:b]


def _world(group=None) -> tuple[int, int]:
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def max_over_ranks(x: float, device=None, group=None) -> float:
    """The largest of every rank's ``x`` (e.g. a device time): a multi-GPU number is the slowest rank's."""
    import torch
    import torch.distributed as dist

    world, _ = _world(group)
    if world == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_in_order(local: Sequence[Any], total: int, group=None, dst: int = 0) -> list | None:
    """Rank ``dst`` gets every rank's results (its :func:`shard` of ``total`` requests) as one list in request
    order; other ranks get None. Each rank must pass exactly its shard's number of results."""
    import torch.distributed as dist

    world, rank = _world(group)
    a, b = shard_bounds(total, world, rank)
    if len(local) != b - a:
        raise ValueError(f"rank {rank}: {len(local)} results for a shard of {b - a} requests")
    if world == 1:
        return list(local)
    parts = [None] * world if rank == dst else None
    dist.gather_object(list(local), parts, dst=dst, group=group)
    if rank != dst:
        return None
    out: list = []
    for r, part in enumerate(parts):
        ra, rb = shard_bounds(total, world, r)
        if len(part) != rb - ra:
            raise RuntimeError(f"rank {r} returned {len(part)} results for {rb - ra} requests")
        out.extend(part)
    return out
