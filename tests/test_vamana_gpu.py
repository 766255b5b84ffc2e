"""GPU Vamana builder (``qv_vamana_gpu``): the host construction step for step.

The host builder (csrc/index_build.cpp) restates the published Vamana
algorithm; the GPU one must produce the same graph, degrees and medoid for
the same seed -- the parity anchor of the build row, since the reference's
own builder (DiskANN) is not in the repository.  Graph quality itself is
checked by the recall of a search over the built index against brute force.
"""
from __future__ import annotations

import numpy as np
import pytest


def test_vamana_gpu_argument_checks_without_gpu():
    import ctypes as C
    from quiver_b200 import _lib
    lib = _lib.engine_lib()
    med = C.c_int64(0)
    assert lib.qv_vamana_gpu(None, 10, 8, 0, 8, 16, 1.2, 2, 0, 0, None, None, C.byref(med)) == 1
    buf = np.zeros((10, 8), dtype=np.uint8)
    g = np.zeros((10, 200), dtype=np.int32)
    d = np.zeros(10, dtype=np.int32)
    assert lib.qv_vamana_gpu(buf.ctypes.data, 10, 8, 0, 200, 16, 1.2, 2, 0, 0, g.ctypes.data, d.ctypes.data,
                             C.byref(med)) == 1  # R above 128
    assert b"R <=" in lib.qv_last_error()


def test_pq_encode_gpu_argument_checks_without_gpu():
    """Chunk offsets are checked before any device call; chunks wider than 64 dims are refused."""
    import ctypes as C
    from quiver_b200 import _lib
    lib = _lib.engine_lib()
    base = np.zeros((4, 130), dtype=np.uint8)
    piv = np.zeros((256, 130), dtype=np.float32)
    cen = np.zeros(130, dtype=np.float32)
    codes = np.zeros((4, 2), dtype=np.uint8)

    def call(offs):
        offs = np.asarray(offs, dtype=np.int32)
        return lib.qv_pq_encode_gpu(base.ctypes.data, 4, 130, _lib.QV_UINT8, len(offs) - 1, piv.ctypes.data,
                                    cen.ctypes.data, offs.ctypes.data, 0, codes.ctypes.data)
    assert call([0, 65, 130]) == _lib.QV_ERR_UNSUPPORTED
    assert b"wider than 64" in lib.qv_last_error()
    assert call([0, 70, 60]) == _lib.QV_ERR_INVALID_ARG
    assert b"chunk offsets" in lib.qv_last_error()
    assert call([0, 64, 131]) == _lib.QV_ERR_INVALID_ARG
    assert lib.qv_pq_encode_gpu(None, 4, 130, _lib.QV_UINT8, 2, None, None, None, 0, None) == _lib.QV_ERR_INVALID_ARG


CASES = [
    # (dtype, n, dim, centers, sigma, R, L, seed)
    ("uint8", 6000, 64, 12, 20.0, 32, 48, 3),
    ("uint8", 20000, 128, 20, 20.0, 64, 100, 5),
    ("uint8", 3000, 50, 6, 25.0, 100, 110, 7),   # odd dim (no 16-byte path), R > 64
    ("float", 4000, 48, 10, 0.1, 32, 48, 4),
    ("float", 5000, 96, 10, 0.1, 64, 100, 6),
]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,n,dim,centers,sigma,R,L,seed", CASES)
def test_gpu_graph_equals_host_graph(dtype, n, dim, centers, sigma, R, L, seed):
    from quiver_b200 import builder
    base = builder.synth_mixture(seed, n, dim, centers, sigma, dtype)
    g_h, d_h, m_h = builder.vamana(base, R=R, L=L, alpha=1.2, passes=2, seed=seed)
    g_g, d_g, m_g = builder.vamana_gpu(base, R=R, L=L, alpha=1.2, passes=2, seed=seed)
    assert m_g == m_h
    np.testing.assert_array_equal(d_g, d_h)
    np.testing.assert_array_equal(g_g, g_h)


@pytest.mark.gpu
def test_gpu_graph_int8_equals_host():
    from quiver_b200 import builder
    rng = np.random.default_rng(9)
    centers = rng.integers(-100, 100, size=(8, 64))
    base = np.clip(centers[rng.integers(0, 8, 4000)] + rng.normal(0, 15, (4000, 64)), -128, 127).astype(np.int8)
    g_h, d_h, m_h = builder.vamana(base, R=32, L=48, alpha=1.2, passes=2, seed=2)
    g_g, d_g, m_g = builder.vamana_gpu(base, R=32, L=48, alpha=1.2, passes=2, seed=2)
    assert m_g == m_h
    np.testing.assert_array_equal(g_g, g_h)


@pytest.mark.gpu
def test_gpu_built_index_searches_like_host_built(tmp_path):
    """Indexes built with the GPU graph and with the host graph give the same search results, and the
    search reaches a sane recall against brute force."""
    from quiver_b200 import Engine, SearchParams, builder
    base = builder.synth_mixture(21, 20000, 128, 20, 20.0, "uint8")
    q = builder.synth_mixture(21, 200, 128, 20, 20.0, "uint8", stream=1).astype(np.float32)
    gt, _ = builder.ground_truth(base, q.astype(np.uint8), 10)
    builder.build_index(tmp_path / "g", base, R=64, L=100, M=32, pq_sample=20000, seed=1, device=0)
    builder.build_index(tmp_path / "h", base, R=64, L=100, M=32, pq_sample=20000, seed=1)
    p = SearchParams(topk=10, ef_search=200, early_exit_policy="none")
    with Engine.open(tmp_path / "g", "uint8") as eng:
        ids_g, d_g, _ = eng.search(q, p)
    with Engine.open(tmp_path / "h", "uint8") as eng:
        ids_h, d_h, _ = eng.search(q, p)
    np.testing.assert_array_equal(ids_g, ids_h)
    np.testing.assert_array_equal(d_g.view(np.uint32), d_h.view(np.uint32))
    recall = np.mean([len(set(a) & set(b)) / 10 for a, b in zip(ids_g, gt)])
    assert recall >= 0.85


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,dim,sigma", [("uint8", 128, 20.0), ("float", 96, 0.1), ("uint8", 37, 30.0)])
def test_gpu_synth_equals_host(dtype, dim, sigma):
    from quiver_b200 import builder
    for stream, row0 in ((0, 0), (1, 12345)):
        h = builder.synth_mixture(7, 3000, dim, 50, sigma, dtype, stream=stream, row0=row0)
        g = builder.synth_mixture(7, 3000, dim, 50, sigma, dtype, stream=stream, row0=row0, device=0)
        np.testing.assert_array_equal(g.view(np.uint8), h.view(np.uint8))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,dim,M", [("uint8", 128, 32), ("float", 96, 32), ("uint8", 50, 12),
                                         ("uint8", 128, 2), ("float", 104, 2)])  # 64- and 52-dim chunks
def test_gpu_pq_encode_equals_host(dtype, dim, M):
    """Chunks wider than 48 dims stage more than the default 48 KB of shared memory per block."""
    from quiver_b200 import builder
    base = builder.synth_mixture(8, 20000, dim, 40, 20.0 if dtype == "uint8" else 0.1, dtype)
    piv, cen, offs = builder.pq_train(base, M, sample=5000, iters=4, seed=1)
    np.testing.assert_array_equal(builder.pq_encode(base, piv, cen, offs, device=0),
                                  builder.pq_encode(base, piv, cen, offs))


@pytest.mark.gpu
def test_gpu_graph_equals_host_graph_with_a_hub(capfd):
    """A point that every new point links to: 60,000 unit vectors in 256 dimensions (nearly equidistant from
    one another) and one vector at the origin, nearer to all of them.  Each batch of 1,200 points sends
    the origin 1,200 new edges, so its reverse-edge pool (R + 1,200 > 1,024) is cut to its 750 nearest by
    the GPU's radix select before pruning, and the near-ties of the distances test the select's order
    (distance bits, then id) against the host's sort."""
    import os
    from quiver_b200 import builder
    rng = np.random.default_rng(31)
    x = rng.normal(size=(60000, 256))
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    x[12345] = 0.0
    base = np.ascontiguousarray(x.astype(np.float32))
    g_h, d_h, m_h = builder.vamana(base, R=16, L=24, alpha=1.2, passes=2, seed=31)
    os.environ["QV_BUILD_LOG"] = "1"
    try:
        g_g, d_g, m_g = builder.vamana_gpu(base, R=16, L=24, alpha=1.2, passes=2, seed=31)
    finally:
        del os.environ["QV_BUILD_LOG"]
    log = capfd.readouterr().err
    largest = [int(ln.rsplit("largest ", 1)[1]) for ln in log.splitlines() if "[vamana_gpu]" in ln]
    assert max(largest) > 1024
    assert m_g == m_h
    np.testing.assert_array_equal(d_g, d_h)
    np.testing.assert_array_equal(g_g, g_h)
