"""Streaming admission (``qv_search_stream``): the reference's persistent-kernel
host loop (src/quiver/search.cu:820-1198).  One launch serves every query
while the host admits ranges as completions allow; results must equal the
batch search's bit for bit, and latency follows the reference's
QueryLatency(ms) definition.  The failure path is exercised without a GPU
fault: the host stops admitting, the waiting workers give up after a short
bounded wait and report an error status, and the engine stays usable.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest


def test_stream_opts_defaults():
    from quiver_b200 import _lib
    o = _lib.StreamOpts()
    _lib.engine_lib().qv_stream_opts_default(C.byref(o))
    assert (o.prefeed, o.admit_min_batch, o.feed_timeout_ms, o.admit_limit) == (-1, 32, 10000, -1)


def test_stream_argument_checks_without_gpu():
    from quiver_b200 import _lib
    lib = _lib.engine_lib()
    o = _lib.SearchOpts()
    lib.qv_search_opts_default(C.byref(o))
    assert lib.qv_search_stream(None, None, 1, 128, C.byref(o), None, None, None, None, None, None) == 1
    assert b"null" in lib.qv_last_error()


def _queries(fx, n):
    reps = -(-n // len(fx["queries"]))
    return np.ascontiguousarray(np.tile(fx["queries"], (reps, 1))[:n])


def _check_stream(eng, q, p, **kw):
    ids, dists, found = eng.search(q, p)
    sids, sdists, sfound, lat, st = eng.search_stream(q, p, **kw)
    np.testing.assert_array_equal(sids, ids)
    np.testing.assert_array_equal(sdists.view(np.uint32), dists.view(np.uint32))
    np.testing.assert_array_equal(sfound, found)
    assert lat.shape == (len(q),) and np.all(lat > 0)
    assert 0 < st.lat_p50_ms <= st.lat_p90_ms <= st.lat_p99_ms <= st.lat_p999_ms <= st.lat_max_ms
    assert st.lat_avg_ms > 0 and st.qps > 0 and st.search_ms > 0
    prefeed = kw.get("prefeed", -1)
    assert st.max_inflight == st.workers + (st.workers if prefeed < 0 else prefeed)
    # the reference's definition: sorted latencies, index n*P/100
    srt = np.sort(lat.astype(np.float64))
    assert abs(srt[len(q) * 99 // 100] - st.lat_p99_ms) <= 1e-3 * max(1.0, st.lat_p99_ms)
    return st


@pytest.mark.gpu
@pytest.mark.parametrize("kw", [{}, {"prefeed": 0}, {"admit_min_batch": 1}, {"prefeed": 7, "admit_min_batch": 500}])
def test_stream_equals_batch_block_kernel(u8_index, kw):
    from quiver_b200 import Engine, SearchParams
    q = _queries(u8_index, 3001)
    with Engine.open(u8_index["dir"], "uint8") as eng:
        st = _check_stream(eng, q, SearchParams(topk=10, ef_search=48, pipe_width=2, early_exit_policy="none"), **kw)
    if st.max_inflight < len(q):
        assert st.admissions >= 2


@pytest.mark.gpu
@pytest.mark.parametrize("policy", ["none", "gpruning"])
def test_stream_equals_batch_warp_kernel(u8_index, policy):
    from quiver_b200 import Engine, SearchParams
    q = _queries(u8_index, 2500)
    with Engine.open(u8_index["dir"], "uint8") as eng:
        _check_stream(eng, q, SearchParams(topk=10, ef_search=40, pipe_width=2, queries_per_block=2,
                                           early_exit_policy=policy), prefeed=0, admit_min_batch=8)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 5, 96])
def test_stream_fewer_queries_than_workers(u8_index, n):
    from quiver_b200 import Engine, SearchParams
    with Engine.open(u8_index["dir"], "uint8") as eng:
        st = _check_stream(eng, _queries(u8_index, n), SearchParams(topk=10, ef_search=48, early_exit_policy="none"))
    assert st.admissions == 1


@pytest.mark.gpu
def test_stream_f32(f32_index):
    from quiver_b200 import Engine, SearchParams
    with Engine.open(f32_index["dir"], "float") as eng:
        _check_stream(eng, _queries(f32_index, 2000), SearchParams(topk=10, ef_search=60, pipe_width=2),
                      prefeed=0, admit_min_batch=4)


@pytest.mark.gpu
def test_stream_feed_timeout_reports_and_recovers(u8_index):
    """The host admits only 100 of 2000 queries; workers bound to later queries
    wait 200 ms, report, and stop; the call fails cleanly and the engine keeps
    working."""
    from quiver_b200 import Engine, QuiverEngineError, SearchParams
    q = _queries(u8_index, 2000)
    p = SearchParams(topk=10, ef_search=48, early_exit_policy="none")
    with Engine.open(u8_index["dir"], "uint8") as eng:
        with pytest.raises(QuiverEngineError, match="not admitted within the feed timeout"):
            eng.search_stream(q, p, admit_limit=100, feed_timeout_ms=200)
        ids, dists, _ = eng.search(q[:64], p)
        sids, sdists, *_ = eng.search_stream(q[:64], p)
    np.testing.assert_array_equal(sids, ids)
    np.testing.assert_array_equal(sdists.view(np.uint32), dists.view(np.uint32))


@pytest.mark.gpu
def test_stream_with_visited_filter_and_nav_off(u8_index):
    """Modes of the search kernel ride along unchanged: the visited filter under streaming admission."""
    from quiver_b200 import Engine, SearchParams
    with Engine.open(u8_index["dir"], "uint8") as eng:
        _check_stream(eng, _queries(u8_index, 1500),
                      SearchParams(topk=10, ef_search=48, pipe_width=2, visited_filter=True,
                                   early_exit_policy="none"), prefeed=0, admit_min_batch=16)


@pytest.mark.gpu
@pytest.mark.parametrize("ef", [320, 700])
def test_stream_long_lists(u8_index, ef):
    """Streaming at the benchmark's ef and with lists above 512 entries (the long-list kernel's streaming
    instantiation) equals the batch search."""
    from quiver_b200 import Engine, SearchParams
    with Engine.open(u8_index["dir"], "uint8") as eng:
        _check_stream(eng, _queries(u8_index, 1200), SearchParams(topk=10, ef_search=ef, pipe_width=2,
                                                                  early_exit_policy="none"),
                      prefeed=0, admit_min_batch=16)
