"""Index files, the product's C++ reader (qv_index_probe, host only) and the
exported C ABI."""
from __future__ import annotations

import ctypes as C
import re
import struct
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def engine_lib():
    from quiver_b200 import _build, _lib
    _build.build_engine()
    return _lib.engine_lib()


def _probe(engine_lib, d, dtype="uint8"):
    from quiver_b200 import _lib
    info = _lib.IndexInfo()
    rc = engine_lib.qv_index_probe(str(d).encode(), _lib.DTYPE_CODES[dtype], C.byref(info))
    return rc, info, engine_lib.qv_last_error().decode()


def _declared_functions(header: Path) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(q[a-z0-9_]+)\s*\(", text, flags=re.M)))


def test_every_declared_symbol_is_exported(engine_lib):
    from quiver_b200 import _lib
    idx = _lib.index_lib()
    for header, lib in ((REPO / "include" / "quiver_b200.h", engine_lib),
                        (REPO / "include" / "quiver_b200_build.h", idx)):
        names = _declared_functions(header)
        assert len(names) >= 5
        for name in names:
            assert hasattr(lib, name), f"{name} declared in {header.name} but not exported"


def test_python_binding_covers_the_header(engine_lib):
    from quiver_b200 import _lib
    declared = set(_declared_functions(REPO / "include" / "quiver_b200.h"))
    assert declared == set(_lib.ENGINE_SYMBOLS)


def test_python_constants_match_the_header():
    """Every integer #define of the C header has the same value in the Python binding."""
    from quiver_b200 import _lib
    text = (REPO / "include" / "quiver_b200.h").read_text()
    defines = re.findall(r"^#define (QV_[A-Z0-9_]+) \(?(\d+)u?(?: << (\d+))?\)?", text, re.M)
    assert len(defines) >= 20
    for name, value, shift in defines:
        expected = int(value) << int(shift or 0)
        assert getattr(_lib, name, None) == expected, f"{name}: header {expected}, binding {getattr(_lib, name, None)}"


def test_library_loads_without_gpu(engine_lib):
    assert engine_lib.qv_version().decode().startswith("quiver-b200")


def test_probe_reads_built_index(engine_lib, u8_index, f32_index):
    for fx, elem in ((u8_index, 1), (f32_index, 4)):
        rc, info, msg = _probe(engine_lib, fx["dir"], fx["dtype"])
        assert rc == 0, msg
        n, dim = fx["base"].shape
        assert (info.num_points, info.dim, info.max_degree, info.num_chunks) == (n, dim, 64, 32)
        assert info.data_size == dim * elem
        assert info.node_size == dim * elem + 4 * 65
        assert info.nodes_per_page == 4096 // info.node_size
        assert info.num_pages == -(-n // info.nodes_per_page)


def test_writer_reader_round_trip(u8_index):
    from quiver_b200 import formats
    from oracle import pyoracle
    d = u8_index["dir"]
    lay = formats.read_disk_index_header(d / "ann_disk.index", "uint8")
    ix = pyoracle.load_index(d, "uint8")
    base = u8_index["base"]
    for v in (0, 1, lay.nodes_per_page, base.shape[0] - 1):
        np.testing.assert_array_equal(ix.vector(v), base[v])
        nb = ix.neighbors(v)
        assert len(nb) <= 64 and (nb < base.shape[0]).all() and v not in nb
        assert len(set(nb.tolist())) == len(nb)
    pq = formats.read_pq(d / "ann")
    np.testing.assert_array_equal(pq["codes"], ix.codes)
    assert pq["chunk_offsets"][0] == 0 and pq["chunk_offsets"][-1] == 128


def test_probe_reads_five_entry_pivot_layout(engine_lib, tmp_path, u8_index):
    """nr = 5 files carry a rearrangement block; chunk offsets then sit at index 3
    (pq_search.cu:74-82)."""
    from quiver_b200 import formats
    src = u8_index["dir"]
    d = tmp_path / "nr5"
    d.mkdir()
    (d / "ann_disk.index").write_bytes((src / "ann_disk.index").read_bytes())
    (d / "ann_pq_compressed.bin").write_bytes((src / "ann_pq_compressed.bin").read_bytes())
    pq = formats.read_pq(src / "ann")
    blobs = [pq["pivots"].astype("<f4"), pq["centroid"].astype("<f4").reshape(-1, 1),
             np.arange(128, dtype="<u4").reshape(-1, 1), pq["chunk_offsets"].astype("<i4").reshape(-1, 1)]
    offs = [4096]
    for b in blobs:
        offs.append(offs[-1] + 8 + b.nbytes)
    with (d / "ann_pq_pivots.bin").open("wb") as f:
        meta = struct.pack("<ii", 5, 1) + struct.pack("<5Q", *offs)
        f.write(meta + b"\0" * (4096 - len(meta)))
        for b in blobs:
            f.write(struct.pack("<ii", *b.shape) + b.tobytes())
    rc, info, msg = _probe(engine_lib, d)
    assert rc == 0, msg
    assert info.num_chunks == 32


def test_probe_accepts_symlinked_disk_index(engine_lib, tmp_path, u8_index):
    """search_setup_test.cpp:107-113: a symlinked *_disk.index is discovered."""
    d = tmp_path / "sym"
    d.mkdir()
    target = tmp_path / "ann.index"
    target.write_bytes((u8_index["dir"] / "ann_disk.index").read_bytes())
    (d / "deep1b_disk.index").symlink_to(target)
    for name in ("ann_pq_pivots.bin", "ann_pq_compressed.bin"):
        (d / name).write_bytes((u8_index["dir"] / name).read_bytes())
    rc, info, msg = _probe(engine_lib, d)
    assert rc == 0, msg


def test_probe_errors(engine_lib, tmp_path, u8_index):
    rc, _, msg = _probe(engine_lib, tmp_path / "missing")
    assert rc == 2 and "does not exist or is not a directory" in msg
    d = tmp_path / "two"
    d.mkdir()
    for name in ("a_disk.index", "b_disk.index"):
        (d / name).write_bytes(b"")
    rc, _, msg = _probe(engine_lib, d)
    assert rc == 2 and "Multiple *_disk.index candidates" in msg
    # PQ trained on another dimension
    d = tmp_path / "mismatch"
    d.mkdir()
    (d / "x_disk.index").write_bytes((u8_index["dir"] / "ann_disk.index").read_bytes())
    from quiver_b200 import formats
    formats.write_pq(d / "x", np.zeros((256, 64), np.float32), np.zeros(64, np.float32),
                     np.arange(0, 65, 2, dtype=np.int32), np.zeros((len(u8_index["base"]), 32), np.uint8))
    rc, _, msg = _probe(engine_lib, d)
    assert rc == 3 and "dimension" in msg


def test_plain_read_errors_do_not_touch_cuda(engine_lib):
    """Invalid arguments are rejected before any device call."""
    from quiver_b200 import _lib
    opts = _lib.EngineOpts(b"/nonexistent", 7, b"heap", None, 0, 0, 0)
    h = C.c_void_p()
    assert engine_lib.qv_engine_create(C.byref(opts), C.byref(h)) == 1


@pytest.mark.parametrize("seed", range(12))
def test_sliced_page_writer_equals_whole_build(tmp_path, engine_lib, seed):
    """write_disk_index writes its pages a slice of nodes at a time; for any slice size (forcing partial last
    pages and slice boundaries inside the data) the file equals the whole-array page build, every record
    reads back (vector, degree, the first `degree` ids, zeros after), and the C++ reader agrees on the
    header."""
    from quiver_b200 import _lib, formats
    rng = np.random.default_rng(seed)
    dtype = [np.uint8, np.int8, np.float32][seed % 3]
    dim = int(rng.integers(3, 140))
    R = int(rng.integers(1, 70))
    elem = np.dtype(dtype).itemsize
    if seed % 2 == 0:
        dim = max(4, dim - dim % 4)  # whole 32-bit words: an index the engine loads
    if dim * elem + 4 * (R + 1) > 4096:
        dim = (4096 - 4 * (R + 1)) // elem
    n = int(rng.integers(1, 400))
    if dtype == np.float32:
        data = rng.standard_normal((n, dim)).astype(np.float32)
    else:
        lim = np.iinfo(dtype)
        data = rng.integers(lim.min, lim.max + 1, size=(n, dim)).astype(dtype)
    degree = rng.integers(0, R + 1, size=n).astype(np.int32)
    graph = np.full((n, R), -1, dtype=np.int32)
    for v in range(n):
        graph[v, :degree[v]] = rng.integers(0, n, size=degree[v])
    medoid = int(rng.integers(0, n))
    d = tmp_path / "ix"
    d.mkdir()
    lay = formats.write_disk_index(d / "ann_disk.index", data, graph, degree, medoid, R,
                                   nodes_per_slice=int(rng.integers(1, 60)))
    whole, node_size, npp = formats.build_pages(data, graph, degree, R)
    assert (lay.node_size, lay.nodes_per_page, lay.num_pages) == (node_size, npp, whole.shape[0])
    assert (d / "ann_disk.index").stat().st_size == 4096 * (lay.num_pages + 1)
    pages = formats.read_pages(d / "ann_disk.index", lay.num_pages)
    np.testing.assert_array_equal(pages, whole)
    dsize = dim * elem
    for v in range(n):
        rec = pages[v // npp, (v % npp) * node_size:(v % npp + 1) * node_size]
        np.testing.assert_array_equal(rec[:dsize].view(dtype), data[v])
        deg = int(rec[dsize:dsize + 4].view("<u4")[0])
        assert deg == degree[v]
        ids = rec[dsize + 4:].view("<u4")
        np.testing.assert_array_equal(ids[:deg], graph[v, :deg])
        assert not ids[deg:].any()
    dt_name = {np.uint8: "uint8", np.int8: "int8", np.float32: "float"}[dtype]
    hdr = formats.read_disk_index_header(d / "ann_disk.index", dt_name)
    assert (hdr.num_points, hdr.dim, hdr.medoid, hdr.max_degree) == (n, dim, medoid, R)
    M = 1
    formats.write_pq(d / "ann", np.zeros((256, dim), np.float32), np.zeros(dim, np.float32),
                     np.array([0, dim], np.int32), np.zeros((n, M), np.uint8))
    rc, info, msg = _probe(engine_lib, d, dt_name)
    if dsize % 4:
        # the ids after the vector are 32-bit words: a record whose vector is not a whole number of words
        # would put them off alignment, so the engine refuses the index rather than load it
        assert rc == _lib.QV_ERR_BAD_INDEX and "4-byte aligned" in msg
        return
    assert rc == 0, msg
    assert (info.num_points, info.dim, info.max_degree, info.node_size, info.nodes_per_page, info.num_pages,
            info.medoid) == (n, dim, R, node_size, npp, lay.num_pages, medoid)
