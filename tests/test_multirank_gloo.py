"""The N > 1 host path on CPU: two gloo ranks shard a query set, search their
slices, time with max over ranks and gather results on rank 0.  The search
itself is the oracle here (no GPU on this host); the check is that the
sharded run reproduces the single-rank results row for row."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, index_dir: str, queries: np.ndarray, out: dict):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "quiver-ae_b200"), str(root)]
    import torch.distributed as dist
    from oracle import pyoracle
    from quiver_b200 import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    ix = pyoracle.load_index(index_dir, "uint8")
    start, n = shard.strong_rows(rank, world, len(queries))
    mine = pyoracle.search(ix, queries[start:start + n], topk=10, ef_search=30, pipe_width=2)
    elapsed = float(rank + 1)  # stand-in per-rank duration
    tmax = shard.reduce_max(elapsed)
    ids = shard.gather_rows(mine["ids"], len(queries))
    if rank == 0:
        out["ids"] = ids
        out["tmax"] = tmax
    dist.barrier()
    dist.destroy_process_group()


def test_strong_rows_cover_exactly_once():
    from quiver_b200 import shard
    for total in (0, 1, 7, 10_000, 10_001):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                s, n = shard.strong_rows(r, world, total)
                seen.extend(range(s, s + n))
            assert seen == list(range(total))
    assert shard.weak_rows(3, 10_000) == (30_000, 10_000)


def test_two_gloo_ranks_match_single_rank(u8_index):
    from oracle import pyoracle
    q = u8_index["queries"][:37]
    ix = pyoracle.load_index(u8_index["dir"], "uint8")
    ref = pyoracle.search(ix, q, topk=10, ef_search=30, pipe_width=2)
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(2, _free_port(), str(u8_index["dir"]), q, out), nprocs=2, join=True)
        np.testing.assert_array_equal(out["ids"], ref["ids"])
        assert out["tmax"] == 2.0
