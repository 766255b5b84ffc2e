"""A hand-checkable index: 8 points on a line, chain graph, exact PQ.

x_i = (10i, 10i, 10i, 10i) as uint8, node i linked to i-1 and i+1, medoid 3,
centroid 0, one PQ chunk whose pivot j < 8 is x_j and code(i) = i, so the ADC
distance equals the exact squared L2 and every step of the walk can be
traced by hand (tests/test_oracle_kats.py spells the trace out).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np


def write_chain_index(d: Path) -> Path:
    from quiver_b200 import formats
    d.mkdir(parents=True, exist_ok=True)
    n, dim, R = 8, 4, 2
    data = np.repeat((np.arange(n) * 10).astype(np.uint8)[:, None], dim, axis=1)
    graph = np.full((n, R), -1, dtype=np.int32)
    degree = np.zeros(n, dtype=np.int32)
    for i in range(n):
        nb = [j for j in (i - 1, i + 1) if 0 <= j < n]
        graph[i, :len(nb)] = nb
        degree[i] = len(nb)
    formats.write_disk_index(d / "chain_disk.index", data, graph, degree, medoid=3, R=R)
    pivots = np.full((256, dim), 1000.0, dtype=np.float32)
    pivots[:n] = data.astype(np.float32)
    formats.write_pq(d / "chain", pivots, np.zeros(dim, np.float32), np.array([0, dim], np.int32),
                     np.arange(n, dtype=np.uint8)[:, None])
    return d
