"""Parity at the benchmark's operating point and above it.

The benchmark runs ef_search = 320 at pipe width 2 on config 0.  Lists longer
than 128 entries put three or four list entries in each thread's registers
in the block kernel's group merge, lists longer than 512 entries switch to
the per-record merge, and the many-pair sort runs whenever more than 32 new
pairs survive the filter.  These tests hold every one of those paths to the
oracle bit for bit (ids, distances, found counts, expansion and gather
counts) on the three fixture indexes, and hold the engine to the reference's
own kernel (oracle/_ref, pipe width 1) and to the oracle (pipe width 2) on
the 1M-point config-0 index itself at ef 320.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engines(u8_index, f32_index, odd_index):
    from quiver_b200 import Engine, _build
    _build.build_engine()
    out = {}
    for fx in (u8_index, f32_index, odd_index):
        out[fx["dir"].name] = Engine.open(fx["dir"], fx["dtype"], validate=True)
    yield out
    for e in out.values():
        e.close()


_ORACLES: dict = {}


def _oracle(fx):
    from oracle import pyoracle
    key = str(fx["dir"])
    if key not in _ORACLES:
        _ORACLES[key] = pyoracle.load_index(fx["dir"], fx["dtype"])
    return _ORACLES[key]


def _compare(eng, ix, queries, **kw):
    from oracle import pyoracle
    from quiver_b200 import SearchParams
    p = SearchParams(**kw)
    ids, dists, found, st = eng.search(queries, p, with_stats=True)
    ref = pyoracle.search(ix, queries, topk=p.topk, ef_search=p.ef_search, pipe_width=p.pipe_width,
                          early_exit_policy=p.early_exit_policy)
    np.testing.assert_array_equal(ids, ref["ids"])
    np.testing.assert_array_equal(dists.view(np.uint32), ref["dists"].view(np.uint32))
    np.testing.assert_array_equal(found, ref["found"])
    assert st.expansions == int(ref["steps"].sum())
    assert st.neighbors_scored == int(ref["nbrs"].sum())
    return ids, ref


@pytest.mark.parametrize("W", [1, 2, 4])
@pytest.mark.parametrize("ef", [129, 200, 320, 512])
@pytest.mark.parametrize("policy", ["none", "gpruning"])
def test_u8_large_lists(engines, u8_index, W, ef, policy):
    _compare(engines["u8"], _oracle(u8_index), u8_index["queries"], topk=10, ef_search=ef, pipe_width=W,
             early_exit_policy=policy)


@pytest.mark.parametrize("W", [1, 2, 4])
@pytest.mark.parametrize("ef", [129, 320, 512])
def test_f32_large_lists(engines, f32_index, W, ef):
    _compare(engines["f32"], _oracle(f32_index), f32_index["queries"], topk=10, ef_search=ef, pipe_width=W,
             early_exit_policy="none")


@pytest.mark.parametrize("W", [1, 2, 4])
@pytest.mark.parametrize("ef", [129, 320])
def test_r100_large_lists(engines, odd_index, W, ef):
    """R = 100 (four neighbours per lane, one record per merge group) and M = 12 (runtime code width)."""
    _compare(engines["odd"], _oracle(odd_index), odd_index["queries"], topk=10, ef_search=ef, pipe_width=W,
             early_exit_policy="gpruning")


@pytest.mark.parametrize("ef", [513, 700, 1024, 2048, 4096])
@pytest.mark.parametrize("W", [1, 2])
def test_u8_per_record_merge(engines, u8_index, ef, W):
    """Lists above 512 entries: the per-record merge with the chunked shift."""
    _compare(engines["u8"], _oracle(u8_index), u8_index["queries"][:48], topk=10, ef_search=ef, pipe_width=W,
             early_exit_policy="none")


@pytest.mark.parametrize("W", [1, 2, 4])
@pytest.mark.parametrize("ef", [45, 320, 1024])
@pytest.mark.parametrize("slots", [0, 2])
def test_int8_parity(i8_index, W, ef, slots):
    """Signed 8-bit data (the int8 instantiations of both kernels): exact distances of signed bytes, from
    short lists to lists above 512 entries."""
    from quiver_b200 import Engine
    with Engine.open(i8_index["dir"], "int8", validate=True) as eng:
        ids, _ = _compare(eng, _oracle(i8_index), i8_index["queries"], topk=10, ef_search=ef, pipe_width=W,
                          early_exit_policy="none", queries_per_block=slots)
    if ef >= 320:
        from oracle import pyoracle
        assert pyoracle.calc_recall(ids, i8_index["gt"], 10) > 0.9


@pytest.mark.parametrize("ef", [700, 1024])
def test_warp_kernel_long_lists(engines, u8_index, ef):
    """The one-warp-per-query kernel with lists above 512 entries."""
    _compare(engines["u8"], _oracle(u8_index), u8_index["queries"][:48], topk=10, ef_search=ef, pipe_width=2,
             early_exit_policy="none", queries_per_block=2)


@pytest.mark.parametrize("slots", [2, 4])
def test_warp_kernel_at_operating_point(engines, u8_index, slots):
    """The one-warp-per-query kernel (queries_per_block >= 2) at ef 320 against the oracle."""
    _compare(engines["u8"], _oracle(u8_index), u8_index["queries"], topk=10, ef_search=320, pipe_width=2,
             early_exit_policy="none", queries_per_block=slots)


# ------------------------------------------------ config 0 itself, 1M points --

CONFIG0_QUERIES = 500


@pytest.fixture(scope="module")
def config0():
    """The benchmark's config-0 index (1M x 128 u8, R=64, L=100, alpha=1.2, PQ 32 x 256), built on cuda:0
    (bit-identical to the host build), and the first rows of its query stream."""
    from oracle import pyoracle
    from quiver_b200 import workloads
    w = workloads.CONFIGS["config0"]
    d = workloads.prepare(w, device=0)
    q = workloads.queries(w, rows=CONFIG0_QUERIES).astype(np.float32)
    return {"dir": d, "ix": pyoracle.load_index(d, "uint8"), "q": q, "w": w}


@pytest.mark.parametrize("policy", ["none", "gpruning"])
def test_config0_ef320_w2_matches_oracle(config0, policy):
    """The benchmark's own setting: config 0, ef 320, pipe width 2."""
    from quiver_b200 import Engine
    with Engine.open(config0["dir"], "uint8") as eng:
        _compare(eng, config0["ix"], config0["q"], topk=10, ef_search=320, pipe_width=2,
                 early_exit_policy=policy)


@pytest.mark.parametrize("policy", ["none", "gpruning"])
def test_config0_ef320_w1_matches_reference_kernel(config0, policy):
    """Config 0 at ef 320, pipe width 1: the engine, the oracle and the reference's own persistent kernel
    (compiled from the reference sources into oracle/_ref) return the same ids, distance bits and found
    counts."""
    from oracle import pyoracle, ref_harness
    from quiver_b200 import Engine, SearchParams
    if not ref_harness.available():
        pytest.skip("reference harness not built (needs the reference sources at build time)")
    ref = ref_harness.run(config0["ix"], config0["q"], topk=10, ef_search=320, early_exit_policy=policy,
                          num_blocks=128, timeout_s=300.0)
    with Engine.open(config0["dir"], "uint8") as eng:
        ids, dists, found = eng.search(config0["q"], SearchParams(topk=10, ef_search=320, pipe_width=1,
                                                                   early_exit_policy=policy))
    orc = pyoracle.search(config0["ix"], config0["q"], topk=10, ef_search=320, pipe_width=1,
                          early_exit_policy=policy)
    for out in ({"ids": ids, "dists": dists, "found": found}, orc):
        np.testing.assert_array_equal(out["ids"], ref["ids"])
        np.testing.assert_array_equal(out["dists"].view(np.uint32), ref["dists"].view(np.uint32))
        np.testing.assert_array_equal(out["found"], ref["found"])
    np.testing.assert_array_equal(orc["steps"], ref["steps"])


def test_config0_page_store_loads_agree(config0):
    """The 410 MB page store reaches HBM in 64 MB pieces through pinned staging buffers (seven pieces here),
    from the heap or the mmap backend, or whole through host memory when the adjacency is validated first:
    the three engines return the same results."""
    from quiver_b200 import Engine, SearchParams
    p = SearchParams(topk=10, ef_search=100, pipe_width=2, early_exit_policy="none")
    q = config0["q"][:200]
    outs = []
    for kw in ({}, {"memory_backend": "mmap"}, {"validate": True}):
        with Engine.open(config0["dir"], "uint8", **kw) as eng:
            outs.append(eng.search(q, p))
    for o in outs[1:]:
        for a, b in zip(o, outs[0]):
            np.testing.assert_array_equal(a, b)
