"""Recall@k as Quiver reports it (bin/common/recall.hpp:6-62).

For each query, the hits are the result ids found in the set of the first k
ground-truth ids; a result id repeated in a row counts every time it
appears (the reference's std::set lookup per result slot).
"""
from __future__ import annotations

import numpy as np


def per_query_hits(results: np.ndarray, gt: np.ndarray, k: int) -> np.ndarray:
    results = np.asarray(results)[:, :k]
    truth = np.asarray(gt)[: results.shape[0], :k]
    # hit[i, j] = results[i, j] in truth[i, :]
    return (results[:, :, None] == truth[:, None, :]).any(axis=2).sum(axis=1)


def calc_recall(results: np.ndarray, gt: np.ndarray, k: int) -> float:
    hits = per_query_hits(results, gt, k)
    return float(hits.sum()) / float(hits.shape[0] * k)
