"""Synthetic inputs and index construction (host library ``libqv_index.so``).

The reference builds indexes with DiskANN (an empty submodule here), so this
module writes the same files from its own Vamana + PQ implementation, and
generates the seeded Gaussian-mixture data that stands in for SIFT/DEEP.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _lib, formats


def _check(rc: int) -> None:
    if rc != _lib.QV_OK:
        msg = _lib.index_lib().qvb_last_error().decode()
        raise RuntimeError(f"libqv_index error {rc}: {msg}")


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def synth_mixture(seed: int, n: int, dim: int, n_centers: int, sigma: float, data_type: str = "uint8",
                  stream: int = 0, row0: int = 0, nthreads: int = 0, device: int | None = None) -> np.ndarray:
    """Rows [row0, row0+n) of the seeded mixture (stream 0 = base, 1 = queries); on GPU `device`
    when given (the same bits)."""
    dt = formats.NUMPY_DTYPES[data_type]
    out = np.empty((n, dim), dtype=dt)
    if device is not None:
        from . import engine
        engine._check(_lib.engine_lib().qv_synth_mixture_gpu(seed, stream, row0, n, dim, n_centers, sigma,
                                                             _lib.DTYPE_CODES[data_type], _ptr(out), device))
        return out
    _check(_lib.index_lib().qvb_synth_mixture(seed, stream, row0, n, dim, n_centers, sigma,
                                               _lib.DTYPE_CODES[data_type], _ptr(out), nthreads))
    return out


def ground_truth(base: np.ndarray, queries: np.ndarray, k: int, nthreads: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Exact squared-L2 top-k (ties by lower id)."""
    base = np.ascontiguousarray(base)
    queries = np.ascontiguousarray(queries, dtype=base.dtype)
    dtype = {np.dtype(np.uint8): _lib.QV_UINT8, np.dtype(np.int8): _lib.QV_INT8,
             np.dtype(np.float32): _lib.QV_FLOAT}[base.dtype]
    ids = np.empty((queries.shape[0], k), dtype=np.int32)
    dists = np.empty((queries.shape[0], k), dtype=np.float32)
    _check(_lib.index_lib().qvb_ground_truth(_ptr(base), base.shape[0], _ptr(queries), queries.shape[0],
                                              base.shape[1], dtype, k, _ptr(ids), _ptr(dists), nthreads))
    return ids, dists


@dataclass
class BuiltIndex:
    index_dir: Path
    prefix: Path
    data_type: str
    layout: formats.DiskLayout


def vamana(base: np.ndarray, R: int, L: int, alpha: float, passes: int = 2, seed: int = 0,
           nthreads: int = 0) -> tuple[np.ndarray, np.ndarray, int]:
    base = np.ascontiguousarray(base)
    n, dim = base.shape
    dtype = {np.dtype(np.uint8): _lib.QV_UINT8, np.dtype(np.int8): _lib.QV_INT8,
             np.dtype(np.float32): _lib.QV_FLOAT}[base.dtype]
    graph = np.empty((n, R), dtype=np.int32)
    degree = np.empty(n, dtype=np.int32)
    medoid = C.c_int64(0)
    _check(_lib.index_lib().qvb_vamana(_ptr(base), n, dim, dtype, R, L, alpha, passes, seed, nthreads,
                                        _ptr(graph), _ptr(degree), C.byref(medoid)))
    return graph, degree, int(medoid.value)


def pq_train(base: np.ndarray, M: int, sample: int = 100_000, iters: int = 12, seed: int = 0,
             nthreads: int = 0) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    base = np.ascontiguousarray(base)
    n, dim = base.shape
    dtype = {np.dtype(np.uint8): _lib.QV_UINT8, np.dtype(np.int8): _lib.QV_INT8,
             np.dtype(np.float32): _lib.QV_FLOAT}[base.dtype]
    pivots = np.empty((256, dim), dtype=np.float32)
    centroid = np.empty(dim, dtype=np.float32)
    offs = np.empty(M + 1, dtype=np.int32)
    _check(_lib.index_lib().qvb_pq_train(_ptr(base), n, dim, dtype, M, sample, iters, seed, nthreads,
                                          _ptr(pivots), _ptr(centroid), _ptr(offs)))
    return pivots, centroid, offs


def pq_encode(base: np.ndarray, pivots: np.ndarray, centroid: np.ndarray, chunk_offsets: np.ndarray,
              nthreads: int = 0, device: int | None = None) -> np.ndarray:
    base = np.ascontiguousarray(base)
    n, dim = base.shape
    M = len(chunk_offsets) - 1
    dtype = {np.dtype(np.uint8): _lib.QV_UINT8, np.dtype(np.int8): _lib.QV_INT8,
             np.dtype(np.float32): _lib.QV_FLOAT}[base.dtype]
    codes = np.empty((n, M), dtype=np.uint8)
    if device is not None:
        from . import engine
        engine._check(_lib.engine_lib().qv_pq_encode_gpu(
            _ptr(base), n, dim, dtype, M, _ptr(np.ascontiguousarray(pivots, dtype=np.float32)),
            _ptr(np.ascontiguousarray(centroid, dtype=np.float32)),
            _ptr(np.ascontiguousarray(chunk_offsets, dtype=np.int32)), device, _ptr(codes)))
        return codes
    _check(_lib.index_lib().qvb_pq_encode(_ptr(base), n, dim, dtype, M,
                                           _ptr(np.ascontiguousarray(pivots, dtype=np.float32)),
                                           _ptr(np.ascontiguousarray(centroid, dtype=np.float32)),
                                           _ptr(np.ascontiguousarray(chunk_offsets, dtype=np.int32)),
                                           nthreads, _ptr(codes)))
    return codes


def vamana_gpu(base: np.ndarray, R: int, L: int, alpha: float, passes: int = 2, seed: int = 0,
               device: int = 0) -> tuple[np.ndarray, np.ndarray, int]:
    """The same construction as ``vamana`` on a GPU (qv_vamana_gpu): equal graph, degrees and medoid."""
    from . import engine
    base = np.ascontiguousarray(base)
    n, dim = base.shape
    dtype = {np.dtype(np.uint8): _lib.QV_UINT8, np.dtype(np.int8): _lib.QV_INT8,
             np.dtype(np.float32): _lib.QV_FLOAT}[base.dtype]
    graph = np.empty((n, R), dtype=np.int32)
    degree = np.empty(n, dtype=np.int32)
    medoid = C.c_int64(0)
    engine._check(_lib.engine_lib().qv_vamana_gpu(_ptr(base), n, dim, dtype, R, L, alpha, passes, seed, device,
                                                  _ptr(graph), _ptr(degree), C.byref(medoid)))
    return graph, degree, int(medoid.value)


def build_index(index_dir: str | Path, base: np.ndarray, *, R: int = 64, L: int = 100, alpha: float = 1.2,
                M: int = 32, passes: int = 2, pq_sample: int = 100_000, pq_iters: int = 12, seed: int = 0,
                prefix: str = "ann", nthreads: int = 0, device: int | None = None) -> BuiltIndex:
    """Write ``<prefix>_disk.index``, ``<prefix>_pq_pivots.bin`` and ``<prefix>_pq_compressed.bin``.
    device: build the graph and encode the codes on that GPU (the same files as the host build)."""
    index_dir = Path(index_dir)
    index_dir.mkdir(parents=True, exist_ok=True)
    base = np.ascontiguousarray(base)
    data_type = {np.dtype(np.uint8): "uint8", np.dtype(np.int8): "int8", np.dtype(np.float32): "float"}[base.dtype]
    if device is None:
        graph, degree, medoid = vamana(base, R, L, alpha, passes, seed, nthreads)
    else:
        graph, degree, medoid = vamana_gpu(base, R, L, alpha, passes, seed, device)
    layout = formats.write_disk_index(index_dir / f"{prefix}_disk.index", base, graph, degree, medoid, R)
    pivots, centroid, offs = pq_train(base, M, pq_sample, pq_iters, seed, nthreads)
    codes = pq_encode(base, pivots, centroid, offs, nthreads, device=device)
    formats.write_pq(index_dir / prefix, pivots, centroid, offs, codes)
    return BuiltIndex(index_dir, index_dir / prefix, data_type, layout)


def nav_sample(n: int, n_nav: int, seed: int) -> np.ndarray:
    """n_nav distinct base ids, ascending, chosen by a seeded permutation."""
    rng = np.random.Generator(np.random.PCG64(seed + 0x6e6176))
    return np.sort(rng.choice(n, size=min(n_nav, n), replace=False)).astype(np.int32)


def build_nav(nav_dir: str | Path, base: np.ndarray, *, n_nav: int = 0, R: int = 28, L: int = 64,
              alpha: float = 1.2, max_m: int = 32, seed: int = 0, nthreads: int = 0) -> formats.NavGraph:
    """A navigation graph over a sample of the base set, in the reference's nav
    format (src/shared/index/nav_graph.cu:12-73), for the in-kernel entry
    search (src/quiver/kernel_core/inkernel_nav.cuh).

    The reference repository has no producer of these files, so this one is
    ours: a Vamana graph (degree R <= 28, the neighbours the entry search
    reads per node) over n_nav seeded samples (default 1 % of the base, at
    least 1,000), started at the sample's medoid, rows padded to max_m."""
    base = np.ascontiguousarray(base)
    n = base.shape[0]
    if n_nav <= 0:
        n_nav = max(1000, n // 100)
    n_nav = min(n_nav, n)
    if R > 28 or R > max_m:
        raise ValueError("the entry search reads at most 28 neighbours per nav node")
    ids = nav_sample(n, n_nav, seed)
    sub = np.ascontiguousarray(base[ids])
    graph, degree, medoid = vamana(sub, R, L, alpha, 2, seed, nthreads)
    if np.any(degree <= 0):
        raise ValueError("nav graph has a node without neighbours (sample too small)")
    padded = np.full((len(ids), max_m), -1, dtype=np.int32)
    padded[:, :R] = graph
    nav = formats.NavGraph(sub, padded, degree.astype(np.int32), ids, int(medoid), max_m)
    formats.write_nav(nav_dir, nav)
    return nav
