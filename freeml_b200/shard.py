"""Sequence sharding for one process per GPU.

Config 3's sequences are independent, so N ranks split them into contiguous
slices with no collective on the data path (each rank runs its own engine on
its own slice); the host only needs the slice bounds, a barrier, and the
max-over-ranks timing reduction used by bench.py.
"""
from __future__ import annotations


def shard_bounds(total: int, world_size: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's sequences; the first total % world_size ranks
    take one extra sequence."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of {world_size}")
    if total < world_size:
        raise ValueError(f"{total} sequences do not shard over {world_size} ranks")
    base, extra = divmod(total, world_size)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, pg=None, device=None) -> float:
    """The maximum of `value` over all ranks (the value itself without a
    process group)."""
    if pg is None:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())
