"""Python access to the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline leg use this module as the checker; the product never imports it.

It carries its own reader of the index files so that a bug in the product's
reader cannot hide behind an identical bug here.  The reader restates
(paths inside ruc-system/quiver-ae): bin/common/metadata.hpp:15-72 (header),
src/shared/index/pq_search.cu:62-114 (PQ files), src/shared/io/mem_loader.cpp:28-44
(pages = file minus its first 4 KB), bin/common/data_io.hpp:73-133 (queries, GT).
"""
from __future__ import annotations

import ctypes as C
import struct
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
ORC_UINT8, ORC_FLOAT, ORC_INT8 = 0, 1, 2
_DT = {"uint8": (ORC_UINT8, np.uint8, 1), "int8": (ORC_INT8, np.int8, 1), "float": (ORC_FLOAT, np.float32, 4)}


def build(force: bool = False) -> Path:
    """gcc recipe: fp32 exactly as written (no contraction), OpenMP over queries."""
    src = HERE / "oracle.c"
    hdr = HERE / "oracle.h"
    LIB.parent.mkdir(exist_ok=True)
    if force or not LIB.exists() or max(src.stat().st_mtime, hdr.stat().st_mtime) > LIB.stat().st_mtime:
        cmd = ["gcc", "-O3", "-mavx2", "-mfma", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC",
               "-shared", str(src), "-o", str(LIB), "-lm"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    return LIB


class _Index(C.Structure):
    _fields_ = [
        ("num_points", C.c_int64), ("dim", C.c_int64), ("max_degree", C.c_int64), ("node_size", C.c_int64),
        ("data_size", C.c_int64), ("nodes_per_page", C.c_int64), ("num_pages", C.c_int64),
        ("medoid", C.c_int64), ("data_type", C.c_int32), ("num_chunks", C.c_int32),
        ("pages", C.c_void_p), ("codes", C.c_void_p), ("pivots_t", C.c_void_p), ("centroid", C.c_void_p),
        ("chunk_offsets", C.c_void_p),
    ]


class _Params(C.Structure):
    _fields_ = [("topk", C.c_int32), ("ef_search", C.c_int32), ("pipe_width", C.c_int32),
                ("early_exit_policy", C.c_int32), ("gpruning_warmup_steps", C.c_int32),
                ("gpruning_patience", C.c_int32), ("num_threads", C.c_int32), ("visited_filter", C.c_int32),
                ("route_exact", C.c_int32)]


_lib = None


class _Nav(C.Structure):
    _fields_ = [("data", C.c_void_p), ("graph", C.c_void_p), ("mapping", C.c_void_p), ("num_node", C.c_int32),
                ("max_m", C.c_int32), ("start", C.c_int32)]


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(str(LIB))
        _lib.orc_build_lut.argtypes = [C.POINTER(_Index), C.c_void_p, C.c_void_p, C.c_void_p]
        _lib.orc_adc.argtypes = [C.c_void_p, C.c_void_p, C.c_int32]
        _lib.orc_adc.restype = C.c_float
        _lib.orc_exact_l2.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32]
        _lib.orc_exact_l2.restype = C.c_float
        _lib.orc_search.argtypes = [C.POINTER(_Index), C.c_void_p, C.c_int64, C.POINTER(_Params), C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        _lib.orc_search.restype = C.c_int
        _lib.orc_search_nav.argtypes = [C.POINTER(_Index), C.c_void_p, C.c_void_p, C.c_int64, C.POINTER(_Params),
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        _lib.orc_search_nav.restype = C.c_int
        _lib.orc_nav_entry.argtypes = [C.POINTER(_Index), C.POINTER(_Nav), C.c_void_p]
        _lib.orc_nav_entry.restype = C.c_int64
        _lib.orc_calc_recall.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int32]
        _lib.orc_calc_recall.restype = C.c_double
    return _lib


@dataclass
class OracleIndex:
    """Index arrays as the reference's loaders produce them."""
    num_points: int
    dim: int
    max_degree: int
    node_size: int
    data_size: int
    nodes_per_page: int
    num_pages: int
    medoid: int
    data_type: str
    pages: np.ndarray          # [num_pages, 4096] u8
    codes: np.ndarray          # [N, M] u8
    pivots: np.ndarray         # [256, dim] f32 as stored
    centroid: np.ndarray       # [dim] f32
    chunk_offsets: np.ndarray  # [M + 1] i32

    def __post_init__(self):
        self.pivots_t = np.ascontiguousarray(self.pivots.T)  # pq_search.cu:141-147
        self._c = _Index(self.num_points, self.dim, self.max_degree, self.node_size, self.data_size,
                         self.nodes_per_page, self.num_pages, self.medoid, _DT[self.data_type][0],
                         self.codes.shape[1], self.pages.ctypes.data, self.codes.ctypes.data,
                         self.pivots_t.ctypes.data, self.centroid.ctypes.data, self.chunk_offsets.ctypes.data)

    @property
    def num_chunks(self) -> int:
        return self.codes.shape[1]

    def record(self, v: int) -> np.ndarray:
        """Node record bytes (search.cu:240, kernel_helpers.cuh:257)."""
        off = (v % self.nodes_per_page) * self.node_size
        return self.pages[v // self.nodes_per_page, off:off + self.node_size]

    def vector(self, v: int) -> np.ndarray:
        return self.record(v)[: self.data_size].view(_DT[self.data_type][1])

    def neighbors(self, v: int) -> np.ndarray:
        rec = self.record(v)
        deg = int(rec[self.data_size:self.data_size + 4].view("<u4")[0])
        return rec[self.data_size + 4:self.data_size + 4 + 4 * deg].view("<u4").astype(np.int64)


def _read_bin_at(f, off: int, dtype) -> np.ndarray:
    f.seek(off)
    n, d = struct.unpack("<ii", f.read(8))
    return np.fromfile(f, dtype=dtype, count=n * d).reshape(n, d)


def load_index(index_dir: str | Path, data_type: str) -> OracleIndex:
    index_dir = Path(index_dir)
    disk = sorted(p for p in index_dir.iterdir() if p.name.endswith("_disk.index"))
    if len(disk) != 1:
        disk = [index_dir / "disk.index"]
    piv = sorted(p for p in index_dir.iterdir() if p.name.endswith("_pq_pivots.bin"))
    prefix = str(piv[0])[: -len("_pivots.bin")] if len(piv) == 1 else str(index_dir / "pq")
    with open(disk[0], "rb") as f:
        _nr, _nc = struct.unpack("<II", f.read(8))
        n, dim, medoid, max_node_len, npp = struct.unpack("<5Q", f.read(40))
    elem = _DT[data_type][2]
    data_size = dim * elem
    R = (max_node_len - data_size) // 4 - 1
    num_pages = (n + npp - 1) // npp
    with open(disk[0], "rb") as f:
        f.seek(4096)
        pages = np.fromfile(f, dtype=np.uint8, count=num_pages * 4096).reshape(num_pages, 4096)
    with open(prefix + "_pivots.bin", "rb") as f:
        offs_arr = _read_bin_at(f, 0, "<u8").reshape(-1)
        chunk_idx = 3 if len(offs_arr) == 5 else 2
        pivots = _read_bin_at(f, int(offs_arr[0]), "<f4")
        centroid = _read_bin_at(f, int(offs_arr[1]), "<f4").reshape(-1)
        chunk_offsets = _read_bin_at(f, int(offs_arr[chunk_idx]), "<i4").reshape(-1)
    with open(prefix + "_compressed.bin", "rb") as f:
        codes = _read_bin_at(f, 0, np.uint8)
    return OracleIndex(int(n), int(dim), int(R), int(max_node_len), int(data_size), int(npp), int(num_pages),
                       int(medoid), data_type, np.ascontiguousarray(pages), np.ascontiguousarray(codes),
                       np.ascontiguousarray(pivots), np.ascontiguousarray(centroid),
                       np.ascontiguousarray(chunk_offsets, dtype=np.int32))


@dataclass
class OracleNav:
    """A navigation graph as NavGraph::init (src/shared/index/nav_graph.cu:12-73) reads it."""
    data: np.ndarray     # [num_node, dim], base data type
    graph: np.ndarray    # [num_node, max_m] i32, -1 padded
    mapping: np.ndarray  # [num_node] i32
    start: int
    max_m: int

    def __post_init__(self):
        self._c = _Nav(self.data.ctypes.data, self.graph.ctypes.data, self.mapping.ctypes.data,
                       self.graph.shape[0], self.max_m, self.start)


def load_nav(index_dir: str | Path, data_type: str) -> OracleNav | None:
    """nav_index / nav_index.data / map.txt in the index directory or its nav/
    child (bin/common/index_discovery.hpp:105-114); None when absent."""
    index_dir = Path(index_dir)
    nav_dir = next((d for d in (index_dir, index_dir / "nav") if (d / "nav_index").exists()), None)
    if nav_dir is None:
        return None
    with open(nav_dir / "nav_index.data", "rb") as f:
        n, data_len = struct.unpack("<ii", f.read(8))
        data = np.fromfile(f, dtype=_DT[data_type][1], count=n * data_len).reshape(n, data_len)
    mapping = np.array([int(x) for x in (nav_dir / "map.txt").read_text().split()[:n]], dtype=np.int32)
    raw = np.fromfile(nav_dir / "nav_index", dtype="<i4")
    max_m, start = int(raw[2]), int(raw[3])
    graph = np.full((n, max_m), -1, dtype=np.int32)
    pos = 6
    for i in range(n):
        d = int(raw[pos])
        if not 0 < d <= max_m:
            raise ValueError(f"nav node {i}: degree {d}")
        graph[i, :d] = raw[pos + 1:pos + 1 + d]
        pos += 1 + d
    return OracleNav(np.ascontiguousarray(data), graph, mapping, start, max_m)


def nav_entry(ix: OracleIndex, nav: OracleNav, query: np.ndarray) -> int:
    q = np.ascontiguousarray(query, dtype=np.float32)
    r = int(lib().orc_nav_entry(C.byref(ix._c), C.byref(nav._c), q.ctypes.data))
    if r < 0:
        raise RuntimeError(f"nav entry search failed with {r}")
    return r


def build_lut(ix: OracleIndex, query: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    q = np.ascontiguousarray(query, dtype=np.float32)
    lut = np.empty((ix.num_chunks, 256), dtype=np.float32)
    q2 = np.empty(ix.dim, dtype=np.float32)
    lib().orc_build_lut(C.byref(ix._c), q.ctypes.data, lut.ctypes.data, q2.ctypes.data)
    return lut, q2


def adc(lut: np.ndarray, code: np.ndarray) -> float:
    code = np.ascontiguousarray(code, dtype=np.uint8)
    lut = np.ascontiguousarray(lut, dtype=np.float32)
    return float(np.float32(lib().orc_adc(lut.ctypes.data, code.ctypes.data, code.shape[0])))


def adc_batch(luts: np.ndarray, codes: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """dist[q, i] = sum_j luts[q, j, codes[ids[q, i], j]], summed in chunk order j = 0..M-1 in fp32
    (the scoring loop of src/shared/kernel_helpers.cuh:271-286, vectorised over pairs: each numpy
    float32 add rounds like the scalar loop's).  Ids outside [0, len(codes)) give NaN."""
    luts = np.asarray(luts, dtype=np.float32)
    nq, M = luts.shape[0], codes.shape[1]
    luts = luts.reshape(nq, M, 256)
    ids = np.asarray(ids, dtype=np.int64).reshape(nq, -1)
    ok = (ids >= 0) & (ids < codes.shape[0])
    safe = np.where(ok, ids, 0)
    qi = np.arange(nq)[:, None]
    acc = np.zeros(ids.shape, dtype=np.float32)
    for j in range(M):
        acc = acc + luts[qi, j, codes[safe, j]]
    return np.where(ok, acc, np.float32(np.nan)).astype(np.float32)


def exact_l2(ix: OracleIndex, q2: np.ndarray, v: int) -> float:
    q2 = np.ascontiguousarray(q2, dtype=np.float32)
    vec = np.ascontiguousarray(ix.vector(v))
    return float(np.float32(lib().orc_exact_l2(q2.ctypes.data, vec.ctypes.data, ix.dim, _DT[ix.data_type][0])))


def search(ix: OracleIndex, queries: np.ndarray, *, topk: int = 10, ef_search: int = 30, pipe_width: int = 1,
           early_exit_policy: str = "none", gpruning_warmup_steps: int = 10, gpruning_patience: int = 8,
           num_threads: int = 0, nav: OracleNav | None = None, visited_filter: bool = False,
           route_exact: bool = False) -> dict:
    """The reference walk (pipe lanes completing in lane order).  route_exact (diagnostic, not reference
    behaviour) scores neighbours by exact L2 instead of ADC, to separate PQ error from graph quality."""
    q = np.ascontiguousarray(queries, dtype=np.float32)
    nq = q.shape[0]
    ids = np.empty((nq, topk), dtype=np.int32)
    dists = np.empty((nq, topk), dtype=np.float32)
    found = np.empty(nq, dtype=np.int32)
    steps = np.empty(nq, dtype=np.int32)
    nbrs = np.empty(nq, dtype=np.int64)
    pol = {"none": 0, "gpruning": 2}[early_exit_policy]
    p = _Params(topk, ef_search, pipe_width, pol, gpruning_warmup_steps, gpruning_patience, num_threads,
                1 if visited_filter else 0, 1 if route_exact else 0)
    rc = lib().orc_search_nav(C.byref(ix._c), C.byref(nav._c) if nav is not None else None, q.ctypes.data, nq,
                              C.byref(p), ids.ctypes.data, dists.ctypes.data, found.ctypes.data,
                              steps.ctypes.data, nbrs.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"oracle search failed with {rc}")
    return {"ids": ids, "dists": dists, "found": found, "steps": steps, "nbrs": nbrs}


def calc_recall(results: np.ndarray, gt: np.ndarray, topk: int) -> float:
    results = np.ascontiguousarray(results, dtype=np.int32)
    gt = np.ascontiguousarray(gt, dtype=np.int32)
    return float(lib().orc_calc_recall(results.ctypes.data, gt.ctypes.data, results.shape[0], gt.shape[1], topk))
