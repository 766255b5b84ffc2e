"""The drop-in CLI on a B200: bin/quiver_search, run on an index directory the way the reference's Python
API runs its binary, writes the engine's ids and distances bit for bit, prints the reference's report lines
with the recall of what it wrote, and refuses query files whose header or data is short.  The reference's
own Python package drives it unchanged, and the in-process front end returns what that chain returns."""
from __future__ import annotations

import re
import struct
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cli():
    from quiver_b200 import _build
    _build.build_engine()
    return _build.build_cli()


def _run(cli, *args):
    return subprocess.run([str(cli), *map(str, args)], capture_output=True, text=True, timeout=300)


@pytest.mark.parametrize("admission,page_store", [("stream", "hbm"), ("batch", "hbm"), ("stream", "host")])
def test_cli_writes_the_engine_results(cli, u8_index, tmp_path, admission, page_store):
    from quiver_b200 import Engine, SearchParams, formats
    from quiver_b200.recall import calc_recall
    d = u8_index["dir"]
    prefix = tmp_path / "res"
    r = _run(cli, "--index-dir", d, "--query", d / "queries.u8bin", "--data-type", "uint8", "--topk", 10,
             "--ef-search", 45, "--pipe-width", 2, "--early-exit-policy", "none", "--repeat", 1,
             "--ground-truth", d / "gt.ibin", "--result-prefix", prefix, "--admission", admission,
             "--page-store", page_store)
    assert r.returncode == 0, r.stderr[-2000:]
    ids = formats.read_bin(f"{prefix}_ids.bin", np.int32)
    dists = formats.read_bin(f"{prefix}_distances.bin", np.float32)
    p = SearchParams(topk=10, ef_search=45, pipe_width=2, early_exit_policy="none")
    with Engine.open(d, "uint8") as eng:
        ref_ids, ref_dists, _ = eng.search(u8_index["queries"], p)
    np.testing.assert_array_equal(ids, ref_ids)
    np.testing.assert_array_equal(dists.view(np.uint32), ref_dists.view(np.uint32))
    assert re.search(r"^  QPS: [0-9]+\.[0-9]{2}$", r.stdout, re.M)
    assert re.search(r"^  QueryLatency\(ms\): avg=[0-9.]+ p50=[0-9.]+ p90=[0-9.]+ p99=[0-9.]+", r.stdout, re.M)
    assert f"admission={admission}" in r.stdout and f"page_store={page_store}" in r.stdout
    m = re.search(r"^Recall @ 10: ([0-9.]+)$", r.stdout, re.M)
    assert m and abs(float(m.group(1)) - calc_recall(ids, u8_index["gt"], 10)) < 1e-6


def test_cli_refuses_short_query_files(cli, u8_index, tmp_path):
    d = u8_index["dir"]
    q = u8_index["queries"].astype(np.uint8)
    short = tmp_path / "short.u8bin"
    short.write_bytes(struct.pack("<ii", *q.shape) + q.tobytes()[: q.size // 2])
    r = _run(cli, "--index-dir", d, "--query", short, "--data-type", "uint8", "--repeat", 1)
    assert r.returncode == 1 and "is truncated" in r.stderr
    bad = tmp_path / "bad.u8bin"
    bad.write_bytes(struct.pack("<ii", -1, q.shape[1]))
    r = _run(cli, "--index-dir", d, "--query", bad, "--data-type", "uint8", "--repeat", 1)
    assert r.returncode == 1 and "Invalid header" in r.stderr
    header_only = tmp_path / "h.u8bin"
    header_only.write_bytes(b"\x01\x00")
    r = _run(cli, "--index-dir", d, "--query", header_only, "--data-type", "uint8", "--repeat", 1)
    assert r.returncode == 1 and "Invalid header" in r.stderr


@pytest.mark.parametrize("policy", ["none", "gpruning"])
def test_reference_python_api_through_this_cli(cli, u8_index, reference_quiver, monkeypatch, policy):
    """The whole drop-in chain: the reference's own Python package, unmodified (installed under
    baseline/_ref from the reference sources), finds this CLI through QUIVER_BINARY and runs it; the arrays
    it returns are the engine's own results for the same queries and options."""
    from quiver_b200 import Engine, SearchParams
    monkeypatch.setenv("QUIVER_BINARY", str(cli))
    idx = reference_quiver.IndexQuiver(u8_index["dir"], data_type="uint8")
    ids, dists = idx.search(u8_index["queries"].astype(np.uint8), topk=10, ef_search=45, early_exit_policy=policy)
    p = SearchParams(topk=10, ef_search=45, pipe_width=2, early_exit_policy=policy)
    with Engine.open(u8_index["dir"], "uint8") as eng:
        ref_ids, ref_dists, _ = eng.search(u8_index["queries"], p)
    np.testing.assert_array_equal(ids, ref_ids)
    np.testing.assert_array_equal(dists.view(np.uint32), ref_dists.view(np.uint32))


@pytest.mark.parametrize("policy", ["none", "gpruning"])
def test_in_process_front_end_matches_the_reference_module(cli, u8_index, reference_quiver, monkeypatch, policy):
    """quiver_b200.IndexQuiver (in process, index kept resident) returns what the reference's module returns
    through this CLI, for the same arguments, on two calls in a row; the same holds for float32 queries that
    the front end first narrows to the index's uint8 as the reference does."""
    from quiver_b200 import IndexQuiver
    monkeypatch.setenv("QUIVER_BINARY", str(cli))
    ref = reference_quiver.IndexQuiver(u8_index["dir"], data_type="uint8", pipe_width=4, queries_per_block=2)
    q = u8_index["queries"] + 0.25
    want = ref.search(q, topk=12, ef_search=60, early_exit_policy=policy)
    with IndexQuiver(u8_index["dir"], data_type="uint8", pipe_width=4, queries_per_block=2) as idx:
        for _ in range(2):
            got = idx.search(q, topk=12, ef_search=60, early_exit_policy=policy)
            np.testing.assert_array_equal(got[0], want[0])
            np.testing.assert_array_equal(got[1].view(np.uint32), want[1].view(np.uint32))
        one = idx.search(q[3], topk=12, ef_search=60, early_exit_policy=policy)
        np.testing.assert_array_equal(one[0][0], want[0][3])
