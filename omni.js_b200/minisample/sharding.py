"""Row sharding across ranks: rows are independent (src/generation.js pickToken
is per row), so each rank samples a contiguous block with no collective."""
from __future__ import annotations


def row_shard(B: int, world: int, rank: int) -> tuple[int, int]:
    """[r0, r1) rows of rank `rank` when B rows are split over `world` ranks:
    contiguous blocks of ceil(B / world), the last ones possibly short or empty."""
    if world < 1 or not 0 <= rank < world or B < 0:
        raise ValueError("bad shard arguments")
    per = -(-B // world)
    r0 = min(B, rank * per)
    return r0, min(B, r0 + per)


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of a per-rank value (step time) over the process group."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def sum_over_ranks(value: float, device=None) -> float:
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t)
    return float(t[0])
