"""Pin the oracle: known answers from the reference's own tests, hand-traced
walks, and exact-rounding checks of every fp32 formula it restates."""
from __future__ import annotations

import struct
from fractions import Fraction

import numpy as np
import pytest

from microindex import write_chain_index


# ------------------------------------------------ reference unit-test KATs --

def test_recall_known_answers():
    """bin/common/search_setup_test.cpp:67-81: per-query hits 3 and 1."""
    from oracle import pyoracle
    from quiver_b200.recall import calc_recall, per_query_hits
    results = np.array([[1, 2, 3], [8, 9, 10]], dtype=np.int32)
    gt = np.array([[3, 2, 1, 4], [7, 8, 11, 12]], dtype=np.int32)
    assert per_query_hits(results, gt, 3).tolist() == [3, 1]
    assert pyoracle.calc_recall(results, gt, 3) == pytest.approx(4 / 6)
    assert calc_recall(results, gt, 3) == pytest.approx(4 / 6)


def test_repeated_result_ids_count_each_time():
    """recall.hpp looks every result slot up in the ground-truth set."""
    from oracle import pyoracle
    from quiver_b200.recall import calc_recall
    results = np.array([[5, 5, 9]], dtype=np.int32)
    gt = np.array([[5, 6, 7]], dtype=np.int32)
    assert pyoracle.calc_recall(results, gt, 3) == pytest.approx(2 / 3)
    assert calc_recall(results, gt, 3) == pytest.approx(2 / 3)


def test_page_store_skips_header_page(tmp_path):
    """src/shared/io/mem_loader_test.cpp:22-80: page p of the store is file page p+1."""
    from quiver_b200 import formats
    f = tmp_path / "disk.index"
    with f.open("wb") as out:
        out.write(bytes(4096))
        for p in range(3):
            out.write(bytes([0x40 + p]) * 4096)
    pages = formats.read_pages(f, 3)
    for p in range(3):
        assert (pages[p] == 0x40 + p).all()


def test_starter_page_offset():
    """search_setup_test.cpp:98-106 / search_setup.hpp:131-134: the entry's page
    sits at byte 4096 * (enter_point / nodes_per_page + 1) of the file."""
    npp = 10
    for enter in (0, 9, 10, 123):
        assert 4096 * (enter // npp + 1) == 4096 + (enter // npp) * 4096


# ------------------------------------------------------ hand-traced walks --

@pytest.fixture()
def chain(tmp_path):
    from oracle import pyoracle
    return pyoracle.load_index(write_chain_index(tmp_path / "chain"), "uint8")


def test_chain_walk_w1(chain):
    """Medoid 3, query x_7, ef 2: the list keeps the two best, the walk is
    3 -> 4 -> 5 -> 6 -> 7 (5 expansions) and the top-3 is 7, 6, 5."""
    from oracle import pyoracle
    q = np.full((1, 4), 70, dtype=np.float32)
    r = pyoracle.search(chain, q, topk=3, ef_search=2, pipe_width=1)
    assert r["ids"].tolist() == [[7, 6, 5]]
    assert r["dists"].tolist() == [[0.0, 400.0, 1600.0]]
    assert r["found"].tolist() == [3]
    assert r["steps"].tolist() == [5]
    assert r["nbrs"].tolist() == [2 * 5 - 1]  # node 7 has one neighbour


def test_chain_walk_w2(chain):
    """W=2: the boot seeds lane 1 with node 2; lane 1's walk ends at once and
    the second lane finds no unvisited entry afterwards: 6 expansions."""
    from oracle import pyoracle
    q = np.full((1, 4), 70, dtype=np.float32)
    r = pyoracle.search(chain, q, topk=3, ef_search=2, pipe_width=2)
    assert r["ids"].tolist() == [[7, 6, 5]]
    assert r["steps"].tolist() == [6]


def test_chain_topk_padding(chain):
    """Unfilled result slots keep id -1 and +inf (kernel_q1.cuh:192-195)."""
    from oracle import pyoracle
    q = np.full((1, 4), 0, dtype=np.float32)
    r = pyoracle.search(chain, q, topk=12, ef_search=2, pipe_width=1)
    assert r["found"][0] < 12
    assert (r["ids"][0, r["found"][0]:] == -1).all()
    assert np.isinf(r["dists"][0, r["found"][0]:]).all()


# ----------------------------------------------- exact fp32 rounding checks --

def _round_f32(x: Fraction) -> np.float32:
    """Round an exact rational to the nearest fp32, ties to even."""
    c = np.float32(float(x))
    best = None
    for cand in (np.nextafter(c, np.float32(-np.inf)), c, np.nextafter(c, np.float32(np.inf))):
        err = abs(Fraction(float(cand)) - x)
        key = (err, int(np.float32(cand).view(np.uint32)) & 1)
        if best is None or key < best[0]:
            best = (key, cand)
    return np.float32(best[1])


def _fma(a, b, c) -> np.float32:
    return _round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def _add(a, b) -> np.float32:
    return _round_f32(Fraction(float(a)) + Fraction(float(b)))


def _sub(a, b) -> np.float32:
    return _round_f32(Fraction(float(a)) - Fraction(float(b)))


@pytest.fixture(scope="module")
def tiny_float_index(tmp_path_factory):
    from oracle import pyoracle
    from quiver_b200 import builder
    d = tmp_path_factory.mktemp("tiny")
    base = builder.synth_mixture(5, 300, 40, 4, 0.3, "float", stream=0)
    builder.build_index(d, base, R=8, L=16, M=10, pq_sample=300, seed=5)
    return pyoracle.load_index(d, "float"), builder.synth_mixture(5, 4, 40, 4, 0.3, "float", stream=1)


def test_lut_and_q2_follow_fused_semantics(tiny_float_index):
    """pq_device.cuh:9-36: q' = q - c, LUT += fma(d, d), q'' = q' + c."""
    from oracle import pyoracle
    ix, queries = tiny_float_index
    q = queries[0].astype(np.float32)
    lut, q2 = pyoracle.build_lut(ix, q)
    qp = [_sub(q[i], ix.centroid[i]) for i in range(ix.dim)]
    for i in range(ix.dim):
        assert q2[i] == _add(qp[i], ix.centroid[i])
    pt = ix.pivots.T
    for c in range(ix.num_chunks):
        for j in (0, 17, 255):
            acc = np.float32(0.0)
            for i in range(ix.chunk_offsets[c], ix.chunk_offsets[c + 1]):
                d = _sub(qp[i], pt[i, j])
                acc = _fma(d, d, acc)
            assert lut[c, j].view(np.uint32) == acc.view(np.uint32)


def test_adc_is_sequential_sum(tiny_float_index):
    from oracle import pyoracle
    ix, queries = tiny_float_index
    lut, _ = pyoracle.build_lut(ix, queries[1].astype(np.float32))
    for v in (0, 7, 299):
        acc = np.float32(0.0)
        for j in range(ix.num_chunks):
            acc = _add(acc, lut[j, ix.codes[v, j]])
        assert np.float32(pyoracle.adc(lut, ix.codes[v])).view(np.uint32) == acc.view(np.uint32)


def test_exact_l2_warp_tree_order(tiny_float_index):
    """gpu_primitives.cuh:26-44: lane-strided fused sums, shfl_down tree 16..1."""
    from oracle import pyoracle
    ix, queries = tiny_float_index
    _, q2 = pyoracle.build_lut(ix, queries[2].astype(np.float32))
    for v in (3, 150):
        x = ix.vector(v)
        lanes = []
        for lane in range(32):
            acc = np.float32(0.0)
            for i in range(lane, ix.dim, 32):
                d = _sub(q2[i], x[i])
                acc = _fma(d, d, acc)
            lanes.append(acc)
        for off in (16, 8, 4, 2, 1):
            lanes = [_add(lanes[l], lanes[l + off] if l + off < 32 else lanes[l]) for l in range(32)]
        assert np.float32(pyoracle.exact_l2(ix, q2, v)).view(np.uint32) == lanes[0].view(np.uint32)


def test_uint8_exact_l2_is_integer_exact():
    """With integral q'' and uint8 data every partial sum is an exact integer."""
    from oracle import pyoracle
    import ctypes as C
    rng = np.random.default_rng(3)
    for _ in range(20):
        q = rng.integers(0, 256, 128).astype(np.float32)
        x = rng.integers(0, 256, 128).astype(np.uint8)
        got = pyoracle.lib().orc_exact_l2(q.ctypes.data, x.ctypes.data, 128, 0)
        assert got == float(((q.astype(np.int64) - x.astype(np.int64)) ** 2).sum())


def test_exact_routing_diagnostic(u8_index):
    """The oracle's route_exact diagnostic walks the same graph with every neighbour scored by its exact L2:
    result distances are still the exact L2 of the returned ids, and on this well-built fixture the walk
    without PQ error finds at least as many true neighbours as the reference walk."""
    from oracle import pyoracle
    ix = pyoracle.load_index(u8_index["dir"], "uint8")
    q = u8_index["queries"]
    pq = pyoracle.search(ix, q, topk=10, ef_search=24, pipe_width=2, early_exit_policy="none")
    ex = pyoracle.search(ix, q, topk=10, ef_search=24, pipe_width=2, early_exit_policy="none", route_exact=True)
    base = u8_index["base"].astype(np.int64)
    for r in range(len(q)):
        got = ex["ids"][r][ex["ids"][r] >= 0]
        want = ((base[got] - q[r].astype(np.int64)) ** 2).sum(1).astype(np.float32)
        np.testing.assert_array_equal(ex["dists"][r][: len(got)], want)
    r_pq = pyoracle.calc_recall(pq["ids"], u8_index["gt"], 10)
    r_ex = pyoracle.calc_recall(ex["ids"], u8_index["gt"], 10)
    assert r_ex >= r_pq
    assert not np.array_equal(pq["ids"], ex["ids"])


def test_recall_attribution_script_runs_on_the_host(tmp_path):
    """tests/recall_attribution.py (the PQ-versus-exact-routing diagnosis) on a small workload, host only:
    one JSON line per ef with both walks, exact routing at least as good as PQ routing."""
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path
    script = Path(__file__).resolve().parent / "recall_attribution.py"
    env = dict(os.environ, QUIVER_B200_CACHE=str(tmp_path / "cache"))
    res = subprocess.run([sys.executable, str(script), "--config", "config0-20k", "--queries", "200", "--efs",
                          "20,60", "--device", "-1"], capture_output=True, text=True, env=env, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    rows = [json.loads(ln) for ln in res.stdout.splitlines() if ln.startswith("{")]
    walks = [r for r in rows if "ef_search" in r]
    assert [r["ef_search"] for r in walks] == [20, 60]
    for r in walks:
        assert r["exact_routing"]["recall_at_10"] >= r["pq_routing"]["recall_at_10"]
