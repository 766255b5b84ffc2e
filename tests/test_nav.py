"""Nav entry search (rows a5 / f2): files, builder, oracle and engine.

The reference picks each query's entry node with a greedy search on a small
navigation graph when one sits next to the index
(src/quiver/kernel_core/inkernel_nav.cuh:60-201, called at
kernel_q1.cuh:149-202; files read by src/shared/index/nav_graph.cu:12-73).
CPU tests pin the file format, the builder and the oracle's restatement
(against a hand-traced chain, and against golden outputs of the reference's
own kernel with nav, tests/golden/ref_nav_*.npz); GPU tests hold both CUDA
kernels to the oracle bit for bit with nav on.
"""
from __future__ import annotations

import shutil
import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_ref_golden as G  # noqa: E402

NAV_CASES = [(name, s) for name in G.FIXTURES for s in G.NAV_SETTINGS]


def _with_nav(root: Path, index_dir: Path, nav_dir: Path) -> Path:
    """An index directory holding the index's files and a nav/ child."""
    d = root / (index_dir.name + "_nav")
    if not d.exists():
        d.mkdir(parents=True)
        for f in index_dir.iterdir():
            if f.is_file():
                (d / f.name).symlink_to(f.resolve())
        shutil.copytree(nav_dir, d / "nav")
    return d


@pytest.fixture(scope="module")
def u8_nav_index(u8_index, tmp_path_factory):
    from quiver_b200 import builder
    root = tmp_path_factory.mktemp("navidx")
    nav_src = root / "src_nav"
    builder.build_nav(nav_src, u8_index["base"], n_nav=400, seed=5)
    return dict(u8_index, dir=_with_nav(root, u8_index["dir"], nav_src), plain=u8_index["dir"])


@pytest.fixture(scope="module")
def f32_nav_index(f32_index, tmp_path_factory):
    from quiver_b200 import builder
    root = tmp_path_factory.mktemp("navidx")
    nav_src = root / "src_nav"
    builder.build_nav(nav_src, f32_index["base"], n_nav=300, seed=6)
    return dict(f32_index, dir=_with_nav(root, f32_index["dir"], nav_src), plain=f32_index["dir"])


# ------------------------------------------------------------------- CPU --

def test_nav_files_round_trip(tmp_path):
    """formats.write_nav -> formats.read_nav and the oracle's own reader agree."""
    from oracle import pyoracle
    from quiver_b200 import builder, formats
    base = builder.synth_mixture(3, 1500, 64, 15, 20.0, "uint8")
    nav = builder.build_nav(tmp_path / "nav", base, n_nav=150, seed=3)
    assert formats.find_nav_dir(tmp_path) == tmp_path / "nav"
    got = formats.read_nav(tmp_path / "nav", "uint8")
    orc = pyoracle.load_nav(tmp_path, "uint8")
    for a, b in ((got.graph, nav.graph), (orc.graph, nav.graph), (got.data, nav.data), (orc.data, nav.data),
                 (got.mapping, nav.mapping), (orc.mapping, nav.mapping)):
        np.testing.assert_array_equal(a, b)
    assert got.start == orc.start == nav.start and got.max_m == orc.max_m == 32
    raw = np.fromfile(tmp_path / "nav" / "nav_index", dtype="<i4")
    assert raw[2] == 32 and raw[3] == nav.start  # the two header fields the reference reads


def test_builder_nav_properties():
    from quiver_b200 import builder
    base = builder.synth_mixture(4, 3000, 32, 10, 20.0, "uint8")
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        nav = builder.build_nav(Path(d), base, n_nav=300, seed=4)
    n = nav.graph.shape[0]
    assert n == 300 and nav.graph.shape[1] == 32
    assert np.all(nav.degree >= 1) and np.all(nav.degree <= 28)  # the search reads 28 neighbours
    assert np.all(nav.graph[:, 28:] == -1)
    assert 0 <= nav.start < n
    assert np.all(np.diff(nav.mapping) > 0) and nav.mapping.max() < 3000
    np.testing.assert_array_equal(nav.data, base[nav.mapping])
    for i in range(n):
        row = nav.graph[i]
        assert np.all(row[:nav.degree[i]] >= 0) and np.all(row[:nav.degree[i]] < n)
        assert np.all(row[nav.degree[i]:] == -1)


def _chain_case(tmp_path):
    """A chain of 40 nav nodes at x = 10 i on the first of 32 u8 dims; node i
    links to i-1 and i+1; the start is node 0; nav id i maps to base id 3 i."""
    from oracle import pyoracle
    n, dim = 40, 32
    data = np.zeros((n, dim), np.uint8)
    data[:, 0] = np.arange(n) * 5
    graph = np.full((n, 32), -1, np.int32)
    for i in range(n):
        nb = [j for j in (i - 1, i + 1) if 0 <= j < n]
        graph[i, :len(nb)] = nb
    mapping = (np.arange(n) * 3).astype(np.int32)
    return pyoracle.OracleNav(data, graph, mapping, 0, 32), data


def test_oracle_nav_chain_walk(tmp_path):
    """The entry search walks the chain to the node nearest the query."""
    from oracle import pyoracle
    ix = pyoracle.load_index(GOLDEN / "idx_u8", "uint8")  # only its dim (128) and N matter... use 32-d case
    nav, data = _chain_case(tmp_path)
    # a 32-d index shell: the oracle reads dim, data type and N from it
    shell = pyoracle.OracleIndex(num_points=1000, dim=32, max_degree=ix.max_degree, node_size=ix.node_size,
                                 data_size=32, nodes_per_page=ix.nodes_per_page, num_pages=ix.num_pages,
                                 medoid=0, data_type="uint8", pages=ix.pages, codes=ix.codes,
                                 pivots=np.zeros((256, 32), np.float32), centroid=np.zeros(32, np.float32),
                                 chunk_offsets=np.arange(0, 33, 1, dtype=np.int32))
    for target in (0, 1, 7, 23, 39):
        q = np.zeros(32, np.float32)
        q[0] = 5 * target + 1.0  # nearest node is `target`
        assert pyoracle.nav_entry(shell, nav, q) == 3 * target


@pytest.mark.parametrize("name,setting", NAV_CASES, ids=[f"{n}-k{s[0]}-ef{s[1]}-{s[2]}" for n, s in NAV_CASES])
def test_oracle_nav_reproduces_reference_kernel(name, setting):
    """Oracle with nav == the reference kernel with its in-kernel nav (pipe width 1)."""
    from oracle import pyoracle
    from quiver_b200 import formats
    k, ef, pol = setting
    tag = f"k{k}_ef{ef}_{pol}"
    ref = np.load(GOLDEN / f"ref_nav_{name}.npz")
    ix = pyoracle.load_index(GOLDEN / name, G.FIXTURES[name]["dtype"])
    nav = pyoracle.load_nav(G.nav_dir(name), G.FIXTURES[name]["dtype"])
    q = formats.read_bin(GOLDEN / name / "queries.fbin", np.float32)
    out = pyoracle.search(ix, q, topk=k, ef_search=ef, pipe_width=1, early_exit_policy=pol, nav=nav)
    np.testing.assert_array_equal(out["ids"], ref[tag + "_ids"])
    np.testing.assert_array_equal(out["dists"].view(np.uint32), ref[tag + "_dists"].view(np.uint32))
    np.testing.assert_array_equal(out["found"], ref[tag + "_found"])
    np.testing.assert_array_equal(out["steps"], ref[tag + "_steps"])
    # and nav changed the walk: without it the results differ for some query
    plain = pyoracle.search(ix, q, topk=k, ef_search=ef, pipe_width=1, early_exit_policy=pol)
    assert not np.array_equal(plain["steps"], out["steps"]) or not np.array_equal(plain["ids"], out["ids"])


# ------------------------------------------------------------------- GPU --

def _compare_nav(fx, nav_dir_root, **kw):
    from oracle import pyoracle
    from quiver_b200 import Engine, SearchParams
    p = SearchParams(**kw)
    ix = pyoracle.load_index(fx["dir"], fx["dtype"])
    nav = pyoracle.load_nav(fx["dir"], fx["dtype"])
    with Engine.open(fx["dir"], fx["dtype"], validate=True) as eng:
        assert eng.nav_info[0] == nav.graph.shape[0]
        ids, dists, found, st = eng.search(fx["queries"], p, with_stats=True)
    ref = pyoracle.search(ix, fx["queries"], topk=p.topk, ef_search=p.ef_search, pipe_width=p.pipe_width,
                          early_exit_policy=p.early_exit_policy, nav=None if p.skip_nav else nav)
    np.testing.assert_array_equal(ids, ref["ids"])
    np.testing.assert_array_equal(dists.view(np.uint32), ref["dists"].view(np.uint32))
    np.testing.assert_array_equal(found, ref["found"])
    assert st.expansions == int(ref["steps"].sum())
    return ref


@pytest.mark.gpu
@pytest.mark.parametrize("qpb", [1, 2])
@pytest.mark.parametrize("W", [1, 2, 4])
@pytest.mark.parametrize("policy", ["none", "gpruning"])
def test_engine_nav_parity_u8(u8_nav_index, qpb, W, policy):
    """Block kernel (one query per CTA) and warp kernel (2 per CTA), nav on."""
    _compare_nav(u8_nav_index, None, topk=10, ef_search=48, pipe_width=W, queries_per_block=qpb,
                 early_exit_policy=policy)


@pytest.mark.gpu
@pytest.mark.parametrize("qpb", [1, 3])
def test_engine_nav_parity_f32(f32_nav_index, qpb):
    _compare_nav(f32_nav_index, None, topk=10, ef_search=40, pipe_width=2, queries_per_block=qpb,
                 early_exit_policy="none")


@pytest.mark.gpu
def test_engine_skip_nav_is_medoid_start(u8_nav_index):
    from quiver_b200 import Engine, SearchParams
    p = SearchParams(topk=10, ef_search=48, pipe_width=2, early_exit_policy="none", skip_nav=True)
    _compare_nav(u8_nav_index, None, **p.__dict__)
    with Engine.open(u8_nav_index["plain"], "uint8") as plain:
        assert plain.nav_info[0] == 0
        a = plain.search(u8_nav_index["queries"], p)
    with Engine.open(u8_nav_index["dir"], "uint8") as eng:
        b = eng.search(u8_nav_index["queries"], p)
    np.testing.assert_array_equal(a[0], b[0])


@pytest.mark.gpu
def test_engine_set_nav_arrays(u8_nav_index):
    """qv_engine_set_nav with host arrays == the same graph loaded from files; num_node 0 removes it."""
    from oracle import pyoracle
    from quiver_b200 import Engine, SearchParams, QuiverEngineError
    nav = pyoracle.load_nav(u8_nav_index["dir"], "uint8")
    p = SearchParams(topk=10, ef_search=48, pipe_width=2, early_exit_policy="none")
    q = u8_nav_index["queries"]
    with Engine.open(u8_nav_index["dir"], "uint8") as eng:
        want = eng.search(q, p)
    with Engine.open(u8_nav_index["plain"], "uint8") as eng:
        medoid = eng.search(q, p)
        eng.set_nav(nav.data, nav.graph, nav.mapping, nav.start)
        assert eng.nav_info == (nav.graph.shape[0], 32, nav.start)
        got = eng.search(q, p)
        bad = nav.mapping.copy()
        bad[0] = 10 ** 9  # not a base id
        with pytest.raises(QuiverEngineError):
            eng.set_nav(nav.data, nav.graph, bad, nav.start)
        eng.set_nav(None)
        assert eng.nav_info[0] == 0
        back = eng.search(q, p)
    np.testing.assert_array_equal(got[0], want[0])
    np.testing.assert_array_equal(got[1].view(np.uint32), want[1].view(np.uint32))
    np.testing.assert_array_equal(back[0], medoid[0])


@pytest.mark.gpu
def test_engine_rejects_bad_nav_files(u8_nav_index, tmp_path):
    from quiver_b200 import Engine, QuiverEngineError
    d = tmp_path / "badnav"
    d.mkdir()
    for f in Path(u8_nav_index["plain"]).iterdir():
        if f.is_file():
            (d / f.name).symlink_to(f.resolve())
    shutil.copytree(Path(u8_nav_index["dir"]) / "nav", d / "nav")
    raw = np.fromfile(d / "nav" / "nav_index", dtype="<i4")
    raw[2] = 40  # max_m above 32
    raw.tofile(d / "nav" / "nav_index")
    with pytest.raises(QuiverEngineError, match="max_m"):
        Engine.open(d, "uint8")


@pytest.mark.gpu
@pytest.mark.parametrize("name,setting", NAV_CASES, ids=[f"{n}-k{s[0]}-ef{s[1]}-{s[2]}" for n, s in NAV_CASES])
def test_engine_nav_reproduces_reference_kernel(name, setting, tmp_path):
    from quiver_b200 import Engine, SearchParams, formats
    k, ef, pol = setting
    tag = f"k{k}_ef{ef}_{pol}"
    ref = np.load(GOLDEN / f"ref_nav_{name}.npz")
    d = _with_nav(tmp_path, GOLDEN / name, G.nav_dir(name))
    q = formats.read_bin(GOLDEN / name / "queries.fbin", np.float32)
    with Engine.open(d, G.FIXTURES[name]["dtype"], validate=True) as eng:
        ids, dists, found = eng.search(q, SearchParams(topk=k, ef_search=ef, pipe_width=1, early_exit_policy=pol))
    np.testing.assert_array_equal(ids, ref[tag + "_ids"])
    np.testing.assert_array_equal(dists.view(np.uint32), ref[tag + "_dists"].view(np.uint32))
    np.testing.assert_array_equal(found, ref[tag + "_found"])
