"""Visited-filter mode: a node a query has scheduled for expansion never
re-enters its candidate list.

Not reference behaviour (the reference tracks visited nodes only by bit 31
inside the list, kernel_helpers.cuh:437-474, so a node that falls out of the
list can come back and be expanded again, and its exact distance can enter
the top-k twice); the engine offers it as an option, off by default, and the
oracle restates the same rule so the CUDA path is still checked bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest


def _oracle(fx):
    from oracle import pyoracle
    return pyoracle.load_index(fx["dir"], fx["dtype"])


def test_oracle_visited_mode_properties(u8_index):
    """No repeated ids in any result row; every row the plain search returns
    without repeats is unchanged or differs only past a node it expanded twice."""
    from oracle import pyoracle
    ix = _oracle(u8_index)
    q = u8_index["queries"]
    for W in (1, 2):
        plain = pyoracle.search(ix, q, topk=10, ef_search=40, pipe_width=W, early_exit_policy="none")
        vis = pyoracle.search(ix, q, topk=10, ef_search=40, pipe_width=W, early_exit_policy="none",
                              visited_filter=True)
        for row in vis["ids"]:
            real = row[row >= 0]
            assert len(set(real.tolist())) == len(real)
        # the mode never expands more nodes than the plain walk needs to fill the same list
        assert vis["steps"].sum() <= plain["steps"].sum()


def _compare(fx, **kw):
    from oracle import pyoracle
    from quiver_b200 import Engine, SearchParams
    p = SearchParams(visited_filter=True, **kw)
    with Engine.open(fx["dir"], fx["dtype"], validate=True) as eng:
        ids, dists, found, st = eng.search(fx["queries"], p, with_stats=True)
        ids2, dists2, _ = eng.search(fx["queries"], p)  # a second search reuses the tables (new tags)
    ref = pyoracle.search(_oracle(fx), fx["queries"], topk=p.topk, ef_search=p.ef_search, pipe_width=p.pipe_width,
                          early_exit_policy=p.early_exit_policy, visited_filter=True)
    np.testing.assert_array_equal(ids, ref["ids"])
    np.testing.assert_array_equal(dists.view(np.uint32), ref["dists"].view(np.uint32))
    np.testing.assert_array_equal(found, ref["found"])
    assert st.expansions == int(ref["steps"].sum())
    np.testing.assert_array_equal(ids2, ids)
    np.testing.assert_array_equal(dists2.view(np.uint32), dists.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("W", [1, 2, 4])
@pytest.mark.parametrize("policy", ["none", "gpruning"])
def test_engine_visited_mode_u8(u8_index, W, policy):
    _compare(u8_index, topk=10, ef_search=48, pipe_width=W, early_exit_policy=policy)


@pytest.mark.gpu
def test_engine_visited_mode_f32(f32_index):
    _compare(f32_index, topk=10, ef_search=60, pipe_width=2, early_exit_policy="none")


@pytest.mark.gpu
def test_engine_visited_mode_long_list(u8_index):
    """ef > 512 takes the per-record merge, which applies the same filter."""
    _compare(dict(u8_index, queries=u8_index["queries"][:16]), topk=10, ef_search=600, pipe_width=2,
             early_exit_policy="none")


@pytest.mark.gpu
def test_engine_visited_mode_rejections(u8_index):
    from quiver_b200 import Engine, QuiverEngineError, SearchParams
    with Engine.open(u8_index["dir"], "uint8") as eng:
        with pytest.raises(QuiverEngineError, match="one query per CTA"):
            eng.search(u8_index["queries"][:4], SearchParams(queries_per_block=2, visited_filter=True))
        with pytest.raises(QuiverEngineError, match="visited-filter"):
            eng.search_noalloc(u8_index["queries"][:4], SearchParams(visited_filter=True))
