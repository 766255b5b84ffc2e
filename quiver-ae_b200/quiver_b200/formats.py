"""DiskANN-layout files that Quiver's search reads, as numpy arrays.

Layouts (paths inside ruc-system/quiver-ae):

* ``*_disk.index`` -- page 0 holds the metadata bin read by
  ``parse_diskann_metadata`` (bin/common/metadata.hpp:15-72): u32 nr, u32 nc,
  then u64 N, dim, medoid, max_node_len, nodes_per_sector, num_frozen,
  frozen_id, reorder_flag (+ file size).  Page p+1 holds nodes
  [p*npp, (p+1)*npp); a node record is the vector, u32 degree, u32[R]
  neighbour ids, zero padded (node_size = dim*elem + 4*(R+1)).
* ``*_pq_pivots.bin`` -- a 4x1 u64 offsets bin at 0; pivots [256 x dim] f32,
  centroid [dim x 1] f32 and chunk offsets [(M+1) x 1] i32 at those offsets
  (src/shared/index/pq_search.cu:62-114).
* ``*_pq_compressed.bin`` -- [N x M] u8 codes.
* ``.u8bin`` / ``.i8bin`` / ``.fbin`` / ``.ibin`` -- i32 n, i32 d, row-major data
  (bin/common/data_io.hpp:23-133).
* nav graph directory (``<index>/nav_index`` or ``<index>/nav/nav_index``,
  found as bin/common/index_discovery.hpp:105-114 does), read by
  ``NavGraph::init`` (src/shared/index/nav_graph.cu:12-73):
  ``nav_index`` -- six i32 (the loader uses field 2 = max_m <= 32 and field 3
  = start; this writer puts num_node and data_len in fields 0 and 1, zeros in
  4 and 5), then per node i32 degree d (0 < d <= max_m) and d i32 nav ids;
  ``nav_index.data`` -- i32 num_node, i32 data_len, then num_node x data_len
  vectors in the base data type; ``map.txt`` -- num_node whitespace-separated
  base-graph ids (nav id -> base id).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

PAGE = 4096
NUMPY_DTYPES = {"uint8": np.uint8, "int8": np.int8, "float": np.float32, "float32": np.float32}


@dataclass
class DiskLayout:
    num_points: int
    dim: int
    medoid: int
    node_size: int
    nodes_per_page: int
    data_size: int
    max_degree: int
    num_pages: int


def write_bin(path: str | Path, arr: np.ndarray) -> None:
    arr = np.ascontiguousarray(arr)
    if arr.ndim != 2:
        raise ValueError("bin files hold 2-D arrays")
    with open(path, "wb") as f:
        f.write(struct.pack("<ii", arr.shape[0], arr.shape[1]))
        f.write(arr.tobytes())


def read_bin(path: str | Path, dtype) -> np.ndarray:
    with open(path, "rb") as f:
        n, d = struct.unpack("<ii", f.read(8))
        data = np.fromfile(f, dtype=dtype, count=n * d)
    if data.size != n * d:
        raise ValueError(f"truncated bin file {path}")
    return data.reshape(n, d)


def node_size_for(dim: int, dtype, R: int) -> int:
    return dim * np.dtype(dtype).itemsize + 4 * (R + 1)


def _page_geometry(data: np.ndarray, R: int) -> tuple[int, int, int]:
    data_size = data.shape[1] * data.dtype.itemsize
    node_size = data_size + 4 * (R + 1)
    npp = PAGE // node_size
    if npp < 1:
        raise ValueError("a node record does not fit in a 4 KB page")
    return data_size, node_size, npp


def _pages_of(data: np.ndarray, graph: np.ndarray, degree: np.ndarray, R: int, n0: int, n1: int) -> np.ndarray:
    """Pages holding nodes [n0, n1) (n0 a multiple of nodes-per-page)."""
    data_size, node_size, npp = _page_geometry(data, R)
    m = n1 - n0
    num_pages = (m + npp - 1) // npp
    full = np.zeros((num_pages * npp, node_size), dtype=np.uint8)
    full[:m, :data_size] = np.ascontiguousarray(data[n0:n1]).view(np.uint8).reshape(m, data_size)
    deg = np.asarray(degree[n0:n1])
    full[:m, data_size:data_size + 4] = deg.astype("<u4").view(np.uint8).reshape(m, 4)
    nb = np.where(np.arange(R)[None, :] < deg[:, None], graph[n0:n1, :R], 0).astype("<u4")
    full[:m, data_size + 4:] = nb.view(np.uint8).reshape(m, 4 * R)
    pages = np.zeros((num_pages, PAGE), dtype=np.uint8)
    pages[:, :npp * node_size] = full.reshape(num_pages, npp * node_size)
    return pages


def build_pages(data: np.ndarray, graph: np.ndarray, degree: np.ndarray, R: int) -> tuple[np.ndarray, int, int]:
    """Node records packed into 4 KB pages -> (pages [P x 4096] u8, node_size, npp)."""
    _, node_size, npp = _page_geometry(data, R)
    return _pages_of(data, graph, degree, R, 0, data.shape[0]), node_size, npp


def write_disk_index(path: str | Path, data: np.ndarray, graph: np.ndarray, degree: np.ndarray,
                     medoid: int, R: int, nodes_per_slice: int = 1 << 20) -> DiskLayout:
    """Header page, then the node pages, written a slice of nodes at a time (bounded memory at any n)."""
    n, dim = data.shape
    _, node_size, npp = _page_geometry(data, R)
    num_pages = (n + npp - 1) // npp
    file_size = PAGE * (num_pages + 1)
    meta = [n, dim, medoid, node_size, npp, 0, 0, 0, file_size]
    header = np.zeros(PAGE, dtype=np.uint8)
    hb = struct.pack("<II", len(meta), 1) + struct.pack(f"<{len(meta)}Q", *meta)
    header[:len(hb)] = np.frombuffer(hb, dtype=np.uint8)
    step = max(npp, nodes_per_slice // npp * npp)
    with open(path, "wb") as f:
        header.tofile(f)
        for n0 in range(0, n, step):
            _pages_of(data, graph, degree, R, n0, min(n, n0 + step)).tofile(f)
    return DiskLayout(n, dim, medoid, node_size, npp, dim * data.dtype.itemsize, R, num_pages)


def read_disk_index_header(path: str | Path, data_type: str) -> DiskLayout:
    with open(path, "rb") as f:
        nr, nc = struct.unpack("<II", f.read(8))
        n, dim, medoid, node_size, npp, _, _, _ = struct.unpack("<8Q", f.read(64))
    elem = np.dtype(NUMPY_DTYPES[data_type]).itemsize
    data_size = dim * elem
    R = (node_size - data_size) // 4 - 1
    return DiskLayout(n, dim, medoid, node_size, npp, data_size, R, (n + npp - 1) // npp)


def read_pages(path: str | Path, num_pages: int) -> np.ndarray:
    with open(path, "rb") as f:
        f.seek(PAGE)
        pages = np.fromfile(f, dtype=np.uint8, count=num_pages * PAGE)
    if pages.size != num_pages * PAGE:
        raise ValueError(f"page store of {path} is truncated")
    return pages.reshape(num_pages, PAGE)


def write_pq(prefix: str | Path, pivots: np.ndarray, centroid: np.ndarray, chunk_offsets: np.ndarray,
             codes: np.ndarray) -> None:
    """Write ``<prefix>_pq_pivots.bin`` (4-entry offsets layout) and ``<prefix>_pq_compressed.bin``."""
    pivots = np.ascontiguousarray(pivots, dtype="<f4")
    centroid = np.ascontiguousarray(centroid, dtype="<f4").reshape(-1, 1)
    chunk_offsets = np.ascontiguousarray(chunk_offsets, dtype="<i4").reshape(-1, 1)
    blobs = [pivots, centroid, chunk_offsets]
    offs = [PAGE]
    for b in blobs:
        offs.append(offs[-1] + 8 + b.nbytes)
    with open(f"{prefix}_pq_pivots.bin", "wb") as f:
        meta = struct.pack("<ii", 4, 1) + struct.pack("<4Q", *offs)
        f.write(meta + b"\0" * (PAGE - len(meta)))
        for b in blobs:
            f.write(struct.pack("<ii", b.shape[0], b.shape[1]))
            f.write(b.tobytes())
    write_bin(f"{prefix}_pq_compressed.bin", np.ascontiguousarray(codes, dtype=np.uint8))


def read_pq(prefix: str | Path) -> dict:
    with open(f"{prefix}_pq_pivots.bin", "rb") as f:
        nr, nc = struct.unpack("<ii", f.read(8))
        offs = struct.unpack(f"<{nr}Q", f.read(8 * nr))
        chunk_idx = 3 if nr == 5 else 2

        def at(off, dtype):
            f.seek(off)
            r, c = struct.unpack("<ii", f.read(8))
            return np.fromfile(f, dtype=dtype, count=r * c).reshape(r, c)

        pivots = at(offs[0], "<f4")
        centroid = at(offs[1], "<f4").reshape(-1)
        chunk_offsets = at(offs[chunk_idx], "<i4").reshape(-1)
    codes = read_bin(f"{prefix}_pq_compressed.bin", np.uint8)
    return {"pivots": pivots, "centroid": centroid, "chunk_offsets": chunk_offsets, "codes": codes}


def load_queries_as_float(path: str | Path, repeat: int = 1) -> np.ndarray:
    """bin/common/data_io.hpp:73-108: the element type follows the file name."""
    name = str(path)
    if ".u8bin" in name:
        q = read_bin(path, np.uint8).astype(np.float32)
    elif ".i8bin" in name:
        q = read_bin(path, np.int8).astype(np.float32)
    else:
        q = read_bin(path, np.float32)
    if repeat > 1:
        q = np.tile(q, (repeat, 1))
    return np.ascontiguousarray(q)


@dataclass
class NavGraph:
    data: np.ndarray      # [num_node x dim], base data type
    graph: np.ndarray     # [num_node x max_m] int32, -1 padded
    degree: np.ndarray    # [num_node] int32
    mapping: np.ndarray   # [num_node] int32, nav id -> base id
    start: int
    max_m: int


def find_nav_dir(index_dir: str | Path) -> Path | None:
    """The directory holding nav_index: the index directory or its nav/ child."""
    index_dir = Path(index_dir)
    for d in (index_dir, index_dir / "nav"):
        if (d / "nav_index").exists():
            return d
    return None


def write_nav(nav_dir: str | Path, nav: NavGraph) -> None:
    nav_dir = Path(nav_dir)
    nav_dir.mkdir(parents=True, exist_ok=True)
    n, dim = nav.data.shape
    if not 0 < nav.max_m <= 32:
        raise ValueError("max_m must be in (0, 32]")
    if np.any(nav.degree <= 0) or np.any(nav.degree > nav.max_m):
        raise ValueError("every nav node needs 0 < degree <= max_m")
    with open(nav_dir / "nav_index", "wb") as f:
        f.write(struct.pack("<6i", n, dim, nav.max_m, nav.start, 0, 0))
        for i in range(n):
            d = int(nav.degree[i])
            f.write(struct.pack("<i", d))
            f.write(np.ascontiguousarray(nav.graph[i, :d], dtype=np.int32).tobytes())
    with open(nav_dir / "nav_index.data", "wb") as f:
        f.write(struct.pack("<ii", n, dim))
        f.write(np.ascontiguousarray(nav.data).tobytes())
    (nav_dir / "map.txt").write_text("\n".join(str(int(x)) for x in nav.mapping) + "\n")


def read_nav(nav_dir: str | Path, data_type: str) -> NavGraph:
    nav_dir = Path(nav_dir)
    dt = NUMPY_DTYPES[data_type]
    with open(nav_dir / "nav_index.data", "rb") as f:
        n, dim = struct.unpack("<ii", f.read(8))
        data = np.fromfile(f, dtype=dt, count=n * dim).reshape(n, dim)
    mapping = np.array(( nav_dir / "map.txt").read_text().split()[:n], dtype=np.int32)
    if mapping.size != n:
        raise ValueError(f"map.txt holds {mapping.size} ids for {n} nav nodes")
    raw = np.fromfile(nav_dir / "nav_index", dtype=np.int32)
    max_m, start = int(raw[2]), int(raw[3])
    graph = np.full((n, max_m), -1, dtype=np.int32)
    degree = np.empty(n, dtype=np.int32)
    pos = 6
    for i in range(n):
        d = int(raw[pos])
        if not 0 < d <= max_m:
            raise ValueError(f"nav node {i} has degree {d} outside (0, {max_m}]")
        graph[i, :d] = raw[pos + 1:pos + 1 + d]
        degree[i] = d
        pos += 1 + d
    return NavGraph(data, graph, degree, mapping, start, max_m)
