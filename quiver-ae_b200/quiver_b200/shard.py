"""Query sharding across ranks (one process per GPU).

Each query's search is independent, so N GPUs split the queries with no
exchange on the data path: every rank holds a replica of the index, searches
its own contiguous slice, and only timing (max over ranks) and, when a
caller wants all results on one rank, a gather cross the process group.
"""
from __future__ import annotations

import numpy as np


def weak_rows(rank: int, per_rank: int) -> tuple[int, int]:
    """Weak scaling: rank r searches rows [r * per_rank, (r + 1) * per_rank)."""
    return rank * per_rank, per_rank


def strong_rows(rank: int, world: int, total: int) -> tuple[int, int]:
    """Strong scaling: a fixed query set split into near-equal contiguous slices."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def reduce_max(value: float, device=None) -> float:
    """Max of a per-rank scalar (a duration) over the default process group."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(local: np.ndarray, total: int, device=None) -> np.ndarray | None:
    """Concatenate every rank's strong_rows slice on rank 0 (None elsewhere)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return local
    world, rank = dist.get_world_size(), dist.get_rank()
    width = local.shape[1]
    biggest = strong_rows(0, world, total)[1]
    buf = torch.zeros((biggest, width), dtype=torch.from_numpy(local[:0]).dtype, device=device)
    buf[: local.shape[0]] = torch.from_numpy(local).to(device)
    parts = [torch.zeros_like(buf) for _ in range(world)] if rank == 0 else None
    dist.gather(buf, parts, dst=0)
    if rank != 0:
        return None
    return np.concatenate([parts[r][: strong_rows(r, world, total)[1]].cpu().numpy() for r in range(world)])
