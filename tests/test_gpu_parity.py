"""Search parity: the CUDA engine (through the C ABI) against the CPU oracle.

Bar: identical ids, bit-identical distances (uint8 and float alike, since
every fp32 operation is specified), identical found counts, expansion and
gather counts, for every pipe width, early-exit policy and list size tried.
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


def _oracle(fx):
    from oracle import pyoracle
    return pyoracle.load_index(fx["dir"], fx["dtype"])


def _compare(eng, ix, queries, **kw):
    from oracle import pyoracle
    from quiver_b200 import SearchParams
    p = SearchParams(**kw)
    ids, dists, found, st = eng.search(queries, p, with_stats=True)
    ref = pyoracle.search(ix, queries, topk=p.topk, ef_search=p.ef_search, pipe_width=p.pipe_width,
                          early_exit_policy=p.early_exit_policy, gpruning_warmup_steps=p.gpruning_warmup_steps,
                          gpruning_patience=p.gpruning_patience)
    np.testing.assert_array_equal(ids, ref["ids"])
    np.testing.assert_array_equal(dists.view(np.uint32), ref["dists"].view(np.uint32))
    np.testing.assert_array_equal(found, ref["found"])
    assert st.expansions == int(ref["steps"].sum())
    assert st.neighbors_scored == int(ref["nbrs"].sum())
    return ids, ref


@pytest.mark.parametrize("W", [1, 2, 4])
@pytest.mark.parametrize("ef", [10, 45, 100])
@pytest.mark.parametrize("policy", ["none", "gpruning"])
def test_u8_parity(engines, u8_index, W, ef, policy):
    _compare(engines["u8"], _oracle(u8_index), u8_index["queries"], topk=10, ef_search=ef, pipe_width=W,
             early_exit_policy=policy)


@pytest.mark.parametrize("W", [1, 3])
@pytest.mark.parametrize("ef", [30, 80])
def test_f32_parity(engines, f32_index, W, ef):
    _compare(engines["f32"], _oracle(f32_index), f32_index["queries"], topk=10, ef_search=ef, pipe_width=W,
             early_exit_policy="none")


@pytest.mark.parametrize("W", [1, 2])
def test_generic_paths_parity(engines, odd_index, W):
    """R=100 (four neighbours per lane) and M=12 (runtime code width)."""
    _compare(engines["odd"], _oracle(odd_index), odd_index["queries"], topk=10, ef_search=40, pipe_width=W,
             early_exit_policy="none")


@pytest.mark.parametrize("k", [1, 33, 64])
def test_topk_sizes(engines, u8_index, k):
    """k = 1 and k > 32 exercise both top-k insert paths."""
    _compare(engines["u8"], _oracle(u8_index), u8_index["queries"][:32], topk=k, ef_search=max(k, 40),
             pipe_width=2, early_exit_policy="none")


def test_ef_below_topk(engines, u8_index):
    _compare(engines["u8"], _oracle(u8_index), u8_index["queries"][:32], topk=20, ef_search=8, pipe_width=1,
             early_exit_policy="none")


@pytest.mark.parametrize("slots", [1, 3, 6])
def test_results_independent_of_geometry(engines, u8_index, slots):
    """Query slots per CTA and grid size change the schedule, never the results."""
    from quiver_b200 import SearchParams
    eng = engines["u8"]
    q = u8_index["queries"]
    base = eng.search(q, SearchParams(ef_search=45, pipe_width=2, early_exit_policy="none"))
    alt = eng.search(q, SearchParams(ef_search=45, pipe_width=2, early_exit_policy="none",
                                     queries_per_block=slots, num_blocks=3))
    for a, b in zip(base, alt):
        np.testing.assert_array_equal(a, b)


def test_oversized_slot_request_is_rejected(engines, u8_index):
    """8 slots of ~36 KB exceed the 227 KB CTA limit: a clean QV_ERR_UNSUPPORTED, no launch."""
    from quiver_b200 import QuiverEngineError, SearchParams
    with pytest.raises(QuiverEngineError, match="do not fit"):
        engines["u8"].search(u8_index["queries"], SearchParams(ef_search=45, queries_per_block=8))


def test_single_and_repeated_queries(engines, u8_index):
    from quiver_b200 import SearchParams
    eng = engines["u8"]
    q = u8_index["queries"]
    p = SearchParams(ef_search=45, pipe_width=1, early_exit_policy="none")
    one = eng.search(q[5], p)
    rep = eng.search(np.tile(q[5:6], (50, 1)), p)
    for r in range(50):
        np.testing.assert_array_equal(rep[0][r], one[0][0])
    empty = eng.search(np.zeros((0, q.shape[1]), np.float32), p)
    assert empty[0].shape == (0, 10)


def test_recall_matches_oracle(engines, u8_index):
    from oracle import pyoracle
    ids, ref = _compare(engines["u8"], _oracle(u8_index), u8_index["queries"], topk=10, ef_search=100,
                        pipe_width=2, early_exit_policy="none")
    r_gpu = pyoracle.calc_recall(ids, u8_index["gt"], 10)
    r_ref = pyoracle.calc_recall(ref["ids"], u8_index["gt"], 10)
    assert r_gpu == r_ref
    assert r_gpu > 0.5


def test_host_page_store_parity(u8_index):
    """Pages in pinned host DRAM (read over PCIe) give the same results."""
    from quiver_b200 import Engine, SearchParams
    p = SearchParams(ef_search=45, pipe_width=2, early_exit_policy="gpruning")
    with Engine.open(u8_index["dir"], "uint8", page_store="host") as eh, \
            Engine.open(u8_index["dir"], "uint8", memory_backend="mmap") as ed:
        a = eh.search(u8_index["queries"], p)
        b = ed.search(u8_index["queries"], p)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_search_device_on_torch_streams(engines, u8_index):
    """search_device on CUDA tensors -- on torch's current stream by default (here the legacy default
    stream), or on a stream given -- returns qv_search's results; tensors of the wrong type, layout or size
    are refused before the launch."""
    import torch
    from quiver_b200 import SearchParams
    eng = engines["u8"]
    q = u8_index["queries"][:64]
    p = SearchParams(ef_search=45, pipe_width=2, early_exit_policy="none")
    ids_h, d_h, f_h = eng.search(q, p)
    dq = torch.from_numpy(q).cuda() * 1.0  # written by a torch kernel on the current stream
    nq, k = q.shape[0], p.topk
    for stream in (None, torch.cuda.Stream()):
        d_ids = torch.full((nq, k), -7, dtype=torch.int32, device="cuda")
        d_dists = torch.empty((nq, k), dtype=torch.float32, device="cuda")
        d_found = torch.empty(nq, dtype=torch.int32, device="cuda")
        if stream is None:
            eng.search_device(dq, p, d_ids, d_dists, d_found)
        else:
            stream.wait_stream(torch.cuda.current_stream())
            eng.search_device(dq, p, d_ids, d_dists, d_found, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        eng.check_device_status()
        np.testing.assert_array_equal(d_ids.cpu().numpy(), ids_h)
        np.testing.assert_array_equal(d_dists.cpu().numpy().view(np.uint32), d_h.view(np.uint32))
        np.testing.assert_array_equal(d_found.cpu().numpy(), f_h)
    with pytest.raises(ValueError, match="torch.int32"):
        eng.search_device(dq, p, d_ids.float(), d_dists)
    with pytest.raises(ValueError, match="contiguous"):
        eng.search_device(dq, p, d_ids.t(), d_dists)
    with pytest.raises(ValueError, match="elements"):
        eng.search_device(dq, p, d_ids[:-1], d_dists)
    with pytest.raises(ValueError, match="elements"):
        eng.build_lut(dq, torch.empty((nq, 31, 256), device="cuda"), torch.empty_like(dq))
    with pytest.raises(ValueError, match="elements"):
        eng.exact_l2(dq, torch.zeros(4, dtype=torch.int32, device="cuda"),
                     torch.zeros(5, dtype=torch.int32, device="cuda"), torch.empty(5, device="cuda"))
