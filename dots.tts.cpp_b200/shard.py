"""Utterance sharding across GPUs: independent utterances are the unit, so
the hot path needs no collective.  GPU g of N takes the contiguous slice
[g*n/N, (g+1)*n/N) of the global utterance list; results are concatenated in
rank order.  The only collective is the max-over-ranks of the timer."""
from __future__ import annotations


def shard_range(n_total: int, world: int, rank: int) -> tuple[int, int]:
    if world < 1 or not (0 <= rank < world) or n_total < 0:
        raise ValueError(f"bad shard request n={n_total} world={world} rank={rank}")
    return (rank * n_total) // world, ((rank + 1) * n_total) // world


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Max of a float over all ranks (identity without a process group)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
