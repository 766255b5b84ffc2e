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


def exchange_stripe_handles(own: bytes, group=None) -> list[bytes]:
    """Every rank's stripe handle, in rank order (one all-gather over the process group)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    got: list = [None] * world
    dist.all_gather_object(got, own, group=group)
    return [bytes(h) for h in got]


def open_shared(index_dir, data_type: str, device: int, group=None, **kw):
    """Open an engine on a page store striped over the ranks of `group`: rank r
    holds pages p = r (mod world) in its GPU's HBM and reads the others from
    the ranks that hold them.  World sizes 1, 2, 4 and 8.  Close the engines
    only after a barrier, since every rank reads every other rank's stripe."""
    import torch.distributed as dist
    from .engine import Engine
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    eng = Engine.open(index_dir, data_type, device=device, page_store="shared", num_stripes=world,
                      stripe_rank=rank, **kw)
    try:
        eng.attach_stripes(exchange_stripe_handles(eng.stripe_handle(), group))
    except Exception:
        eng.close()
        raise
    return eng
