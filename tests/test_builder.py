"""Synthetic inputs and the index builder (host library)."""
from __future__ import annotations

import numpy as np
import pytest


def test_mixture_is_deterministic_and_streams_differ():
    from quiver_b200 import builder
    a = builder.synth_mixture(7, 500, 32, 5, 20.0, "uint8", stream=0)
    b = builder.synth_mixture(7, 500, 32, 5, 20.0, "uint8", stream=0)
    np.testing.assert_array_equal(a, b)
    c = builder.synth_mixture(7, 500, 32, 5, 20.0, "uint8", stream=1)
    assert not np.array_equal(a, c)
    # a slice of rows equals the same rows of the full draw
    s = builder.synth_mixture(7, 100, 32, 5, 20.0, "uint8", stream=0, row0=200)
    np.testing.assert_array_equal(s, a[200:300])
    # thread count does not change the values
    t = builder.synth_mixture(7, 500, 32, 5, 20.0, "uint8", stream=0, nthreads=1)
    np.testing.assert_array_equal(t, a)


def test_mixture_shapes_and_statistics():
    from quiver_b200 import builder
    f = builder.synth_mixture(1, 2000, 96, 10, 0.1, "float")
    assert f.dtype == np.float32
    np.testing.assert_allclose(np.linalg.norm(f, axis=1), 1.0, rtol=1e-5)
    u = builder.synth_mixture(1, 2000, 128, 1, 20.0, "uint8")
    # one centre: per-coordinate spread close to sigma (away from the clip edges)
    sd = u.astype(np.float64).std(axis=0)
    assert 15 < np.median(sd) < 22


def test_ground_truth_matches_brute_force():
    from quiver_b200 import builder
    base = builder.synth_mixture(2, 3000, 24, 6, 20.0, "uint8")
    q = builder.synth_mixture(2, 20, 24, 6, 20.0, "uint8", stream=1)
    ids, dists = builder.ground_truth(base, q, 10)
    d = ((q[:, None, :].astype(np.int64) - base[None].astype(np.int64)) ** 2).sum(-1)
    for i in range(q.shape[0]):
        order = np.lexsort((np.arange(base.shape[0]), d[i]))[:10]
        np.testing.assert_array_equal(ids[i], order)
        np.testing.assert_array_equal(dists[i], d[i, order])


def test_vamana_graph_invariants():
    from quiver_b200 import builder
    base = builder.synth_mixture(3, 4000, 32, 8, 20.0, "uint8")
    g, deg, med = builder.vamana(base, 24, 40, 1.2, passes=2, seed=3)
    assert 0 <= med < len(base)
    assert (deg >= 1).all() and (deg <= 24).all()
    for v in range(len(base)):
        nb = g[v, :deg[v]]
        assert (nb >= 0).all() and (nb < len(base)).all()
        assert v not in nb
        assert len(np.unique(nb)) == len(nb)
        assert (g[v, deg[v]:] == -1).all()
    # deterministic across thread counts
    g1, d1, m1 = builder.vamana(base, 24, 40, 1.2, passes=2, seed=3, nthreads=1)
    np.testing.assert_array_equal(g, g1)
    assert m1 == med


def test_vamana_graph_is_navigable():
    """Greedy search on the built graph with exact distances finds the true NN."""
    from quiver_b200 import builder
    base = builder.synth_mixture(4, 3000, 32, 6, 20.0, "uint8")
    q = builder.synth_mixture(4, 50, 32, 6, 20.0, "uint8", stream=1)
    g, deg, med = builder.vamana(base, 32, 64, 1.2, passes=2, seed=4)
    gt, _ = builder.ground_truth(base, q, 1)
    hits = 0
    for i in range(len(q)):
        qv = q[i].astype(np.int64)

        def dist(v):
            return int(((base[v].astype(np.int64) - qv) ** 2).sum())

        cand, seen, expanded = [(dist(med), med)], {med}, set()
        while True:
            nxt = next((v for _, v in cand if v not in expanded), None)
            if nxt is None:
                break
            expanded.add(nxt)
            for u in g[nxt, :deg[nxt]].tolist():
                if u not in seen:
                    seen.add(u)
                    cand.append((dist(u), u))
            cand = sorted(cand)[:64]
        hits += cand[0][1] == gt[i, 0]
    assert hits >= 48


def test_pq_codes_are_nearest_pivots():
    from quiver_b200 import builder
    base = builder.synth_mixture(5, 2000, 16, 4, 20.0, "uint8")
    piv, cen, off = builder.pq_train(base, 4, sample=2000, iters=5, seed=5)
    assert off.tolist() == [0, 4, 8, 12, 16]
    np.testing.assert_allclose(cen, base[:2000].astype(np.float64).mean(0), rtol=1e-5)
    codes = builder.pq_encode(base, piv, cen, off)
    r = base.astype(np.float32) - cen
    for c in range(4):
        sl = slice(off[c], off[c + 1])
        d = ((r[:, None, sl] - piv[None, :, sl]) ** 2).sum(-1)
        best = d.min(1)
        chosen = d[np.arange(len(base)), codes[:, c]]
        np.testing.assert_allclose(chosen, best, rtol=1e-5, atol=1e-3)


def test_uneven_chunks():
    from quiver_b200 import builder
    base = builder.synth_mixture(6, 500, 10, 2, 20.0, "uint8")
    _, _, off = builder.pq_train(base, 4, sample=500, iters=2)
    assert off.tolist() == [0, 3, 6, 8, 10]
