"""Python handle on the C ABI engine (include/quiver_b200.h).

``Engine.search`` is the host-buffer call (``qv_search``); ``Engine.search_device``
takes CUDA tensors already resident on the engine's GPU (``qv_search_device``).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _lib, formats


class QuiverEngineError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[qv error {code}] {message}")
        self.code = code


def _check(rc: int) -> None:
    if rc != _lib.QV_OK:
        raise QuiverEngineError(rc, _lib.engine_lib().qv_last_error().decode(errors="replace"))


@dataclass
class SearchParams:
    topk: int = 10
    ef_search: int = 30
    pipe_width: int = 2
    queries_per_block: int = 0
    num_blocks: int = 0
    early_exit_policy: str = "gpruning"
    gpruning_warmup_steps: int = 10
    gpruning_patience: int = 8
    lut_mode: int = _lib.QV_LUT_FP32
    skip_nav: bool = False   # True: entry = medoid even when the engine holds a nav graph
    visited_filter: bool = False  # True: expanded nodes never re-enter the list (not reference behaviour)

    def to_c(self) -> _lib.SearchOpts:
        pol = {"none": _lib.QV_EXIT_NONE, "gpruning": _lib.QV_EXIT_GPRUNING}[self.early_exit_policy]
        return _lib.SearchOpts(self.topk, self.ef_search, self.pipe_width, self.queries_per_block,
                               self.num_blocks, pol, self.gpruning_warmup_steps, self.gpruning_patience,
                               self.lut_mode, 1 if self.skip_nav else 0, 1 if self.visited_filter else 0)


class Engine:
    """One index resident on one GPU."""

    def __init__(self, handle: C.c_void_p, device: int = 0):
        self._h = handle
        self._lib = _lib.engine_lib()
        self.device = device  # the GPU the engine's kernels run on
        i = self.info
        self._dim, self._M = int(i.dim), int(i.num_chunks)

    @classmethod
    def open(cls, index_dir: str | Path, data_type: str = "uint8", *, memory_backend: str = "heap",
             memory_index_file: str | None = None, device: int = 0, page_store: str = "hbm",
             validate: bool = False, stripe_devices: list[int] | None = None, num_stripes: int = 0,
             stripe_rank: int = -1) -> "Engine":
        """page_store: "hbm", "host" (pinned mapped DRAM), "striped" (page p on
        stripe_devices[p % len(stripe_devices)], read by peer loads) or "shared"
        (this process holds stripe `stripe_rank` of `num_stripes`; call
        stripe_handle / attach_stripes -- shard.open_shared does both -- before
        searching)."""
        lib = _lib.engine_lib()
        devs = np.ascontiguousarray(stripe_devices or [], dtype=np.int32)
        opts = _lib.EngineOpts(str(index_dir).encode(), _lib.DTYPE_CODES[data_type], memory_backend.encode(),
                               memory_index_file.encode() if memory_index_file else None, device,
                               {"hbm": _lib.QV_PAGES_HBM, "host": _lib.QV_PAGES_HOST,
                                "striped": _lib.QV_PAGES_STRIPED, "shared": _lib.QV_PAGES_SHARED}[page_store],
                               1 if validate else 0, num_stripes if page_store == "shared" else len(devs),
                               C.c_void_p(devs.ctypes.data) if len(devs) else None, stripe_rank)
        h = C.c_void_p()
        _check(lib.qv_engine_create(C.byref(opts), C.byref(h)))
        return cls(h, device)

    @classmethod
    def from_arrays(cls, *, data_type: str, num_points: int, dim: int, node_size: int, nodes_per_page: int,
                    medoid: int, pages: np.ndarray, codes: np.ndarray, pivots: np.ndarray, centroid: np.ndarray,
                    chunk_offsets: np.ndarray, device: int = 0, page_store: str = "hbm") -> "Engine":
        lib = _lib.engine_lib()
        keep = [np.ascontiguousarray(pages, dtype=np.uint8), np.ascontiguousarray(codes, dtype=np.uint8),
                np.ascontiguousarray(pivots, dtype=np.float32), np.ascontiguousarray(centroid, dtype=np.float32),
                np.ascontiguousarray(chunk_offsets, dtype=np.int32)]
        info = _lib.IndexInfo(num_points, dim, 0, node_size, 0, nodes_per_page, 0, medoid,
                              _lib.DTYPE_CODES[data_type], len(chunk_offsets) - 1)
        arr = _lib.IndexArrays(info, *[C.c_void_p(a.ctypes.data) for a in keep])
        h = C.c_void_p()
        _check(lib.qv_engine_create_from_arrays(C.byref(arr), device,
                                                {"hbm": _lib.QV_PAGES_HBM, "host": _lib.QV_PAGES_HOST}[page_store],
                                                C.byref(h)))
        return cls(h, device)

    def close(self) -> None:
        if self._h:
            self._lib.qv_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_nav(self, data: np.ndarray | None, graph: np.ndarray | None = None, mapping: np.ndarray | None = None,
                start: int = 0) -> None:
        """Replace the nav graph (data [n x dim] of the index's type, graph [n x max_m] int32 -1 padded,
        mapping [n] int32); data=None removes it."""
        if data is None:
            _check(self._lib.qv_engine_set_nav(self._h, None, None, None, 0, 0, 0))
            return
        data = np.ascontiguousarray(data)
        graph = np.ascontiguousarray(graph, dtype=np.int32)
        mapping = np.ascontiguousarray(mapping, dtype=np.int32)
        _check(self._lib.qv_engine_set_nav(self._h, C.c_void_p(data.ctypes.data), C.c_void_p(graph.ctypes.data),
                                           C.c_void_p(mapping.ctypes.data), graph.shape[0], graph.shape[1],
                                           start))

    @property
    def nav_info(self) -> tuple[int, int, int]:
        """(num_node, max_m, start); num_node 0 when the engine has no nav graph."""
        n, m, st = C.c_int32(), C.c_int32(), C.c_int32()
        _check(self._lib.qv_engine_nav_info(self._h, C.byref(n), C.byref(m), C.byref(st)))
        return n.value, m.value, st.value

    @property
    def info(self) -> _lib.IndexInfo:
        i = _lib.IndexInfo()
        _check(self._lib.qv_engine_info(self._h, C.byref(i)))
        return i

    def plan(self, params: SearchParams, nq: int) -> _lib.SearchStats:
        st = _lib.SearchStats()
        o = params.to_c()
        _check(self._lib.qv_plan(self._h, C.byref(o), nq, C.byref(st)))
        return st

    def search(self, queries: np.ndarray, params: SearchParams | None = None, *, out=None,
               with_stats: bool = False):
        """Host buffers in and out: returns (ids [nq,k] i32, dists [nq,k] f32, found [nq] i32[, stats])."""
        params = params or SearchParams()
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim == 1:
            q = q.reshape(1, -1)
        nq, dim = q.shape
        k = params.topk
        if out is None:
            ids = np.empty((nq, k), dtype=np.int32)
            dists = np.empty((nq, k), dtype=np.float32)
            found = np.empty(nq, dtype=np.int32)
        else:
            ids, dists, found = out
        st = _lib.SearchStats()
        o = params.to_c()
        _check(self._lib.qv_search(self._h, C.c_void_p(q.ctypes.data), nq, dim, C.byref(o),
                                   C.c_void_p(ids.ctypes.data), C.c_void_p(dists.ctypes.data),
                                   C.c_void_p(found.ctypes.data), C.byref(st) if with_stats else None))
        if with_stats:
            return ids, dists, found, st
        return ids, dists, found

    def search_timed(self, queries: np.ndarray, params: SearchParams | None = None):
        """qv_search_timed: also returns per-query service latency in ms."""
        params = params or SearchParams()
        q = np.ascontiguousarray(queries, dtype=np.float32)
        nq, dim = q.shape
        ids = np.empty((nq, params.topk), dtype=np.int32)
        dists = np.empty((nq, params.topk), dtype=np.float32)
        found = np.empty(nq, dtype=np.int32)
        ms = np.empty(nq, dtype=np.float32)
        st = _lib.SearchStats()
        o = params.to_c()
        _check(self._lib.qv_search_timed(self._h, C.c_void_p(q.ctypes.data), nq, dim, C.byref(o),
                                         C.c_void_p(ids.ctypes.data), C.c_void_p(dists.ctypes.data),
                                         C.c_void_p(found.ctypes.data), C.c_void_p(ms.ctypes.data), C.byref(st)))
        return ids, dists, found, ms, st

    def stripe_handle(self) -> bytes:
        """CUDA IPC handle of the stripe this process holds (shared page store)."""
        buf = C.create_string_buffer(_lib.QV_STRIPE_HANDLE_BYTES)
        _check(self._lib.qv_engine_stripe_handle(self._h, buf))
        return buf.raw

    def attach_stripes(self, handles: list[bytes]) -> None:
        """Open every other process's stripe (handles in stripe order); the engine can search afterwards."""
        blob = b"".join(handles)
        if any(len(h) != _lib.QV_STRIPE_HANDLE_BYTES for h in handles):
            raise ValueError("every stripe handle is QV_STRIPE_HANDLE_BYTES long")
        _check(self._lib.qv_engine_attach_stripes(self._h, C.c_char_p(blob)))

    def search_stream(self, queries: np.ndarray, params: SearchParams | None = None, *, prefeed: int = -1,
                      admit_min_batch: int = 32, feed_timeout_ms: int = 10000, admit_limit: int = -1):
        """qv_search_stream: one persistent launch, queries admitted by the host
        as completions allow (the reference's streaming loop).  Returns (ids,
        dists, found, latency_ms, stats) with the reference's QueryLatency
        definition (admission to observed completion, in completion order)."""
        params = params or SearchParams()
        q = np.ascontiguousarray(queries, dtype=np.float32)
        nq, dim = q.shape
        ids = np.empty((nq, params.topk), dtype=np.int32)
        dists = np.empty((nq, params.topk), dtype=np.float32)
        found = np.empty(nq, dtype=np.int32)
        lat = np.empty(nq, dtype=np.float32)
        so = _lib.StreamOpts(prefeed, admit_min_batch, feed_timeout_ms, admit_limit)
        st = _lib.StreamStats()
        o = params.to_c()
        _check(self._lib.qv_search_stream(self._h, C.c_void_p(q.ctypes.data), nq, dim, C.byref(o), C.byref(so),
                                          C.c_void_p(ids.ctypes.data), C.c_void_p(dists.ctypes.data),
                                          C.c_void_p(found.ctypes.data), C.c_void_p(lat.ctypes.data),
                                          C.byref(st)))
        return ids, dists, found, lat, st

    def search_noalloc(self, queries: np.ndarray, params: SearchParams | None = None):
        """qv_search_noalloc: the same search with no device allocation on the call
        path (its scratch is a fixed 4 MiB device array); returns (ids, dists, found)."""
        params = params or SearchParams()
        q = np.ascontiguousarray(queries, dtype=np.float32)
        nq, dim = q.shape
        ids = np.empty((nq, params.topk), dtype=np.int32)
        dists = np.empty((nq, params.topk), dtype=np.float32)
        found = np.empty(nq, dtype=np.int32)
        o = params.to_c()
        _check(self._lib.qv_search_noalloc(self._h, C.c_void_p(q.ctypes.data), nq, dim, C.byref(o),
                                           C.c_void_p(ids.ctypes.data), C.c_void_p(dists.ctypes.data),
                                           C.c_void_p(found.ctypes.data)))
        return ids, dists, found

    def search_host_ptrs(self, q_ptr: int, nq: int, dim: int, params: SearchParams, ids_ptr: int,
                         dists_ptr: int, found_ptr: int | None = None) -> None:
        """qv_search on raw host pointers (e.g. pinned torch tensors)."""
        o = params.to_c()
        _check(self._lib.qv_search(self._h, C.c_void_p(q_ptr), nq, dim, C.byref(o), C.c_void_p(ids_ptr),
                                   C.c_void_p(dists_ptr), C.c_void_p(found_ptr) if found_ptr else None, None))

    def _arg(self, t, name: str, dtype, numel: int | None = None):
        """Device pointer of a contiguous CUDA tensor on the engine's GPU, after checking its type and size."""
        import torch
        if t is None:
            return None
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.device.index != self.device:
            raise ValueError(f"{name} must be a CUDA tensor on cuda:{self.device}")
        if t.dtype != dtype:
            raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        if numel is not None and t.numel() != numel:
            raise ValueError(f"{name} must hold {numel} elements, got {t.numel()}")
        return C.c_void_p(t.data_ptr())

    def _queries(self, t, name: str) -> int:
        import torch
        if not isinstance(t, torch.Tensor) or t.dim() != 2 or t.shape[1] != self._dim:
            raise ValueError(f"{name} must be [nq, {self._dim}]")
        return t.shape[0]

    def search_device(self, d_queries, params: SearchParams, d_ids, d_dists, d_found=None, d_steps=None,
                      d_nbrs=None, stream=None) -> None:
        """Enqueue a search on CUDA tensors (torch) without synchronising.

        d_queries float32 [nq, dim]; d_ids int32 and d_dists float32 [nq, topk];
        d_found, d_steps int32 [nq] and d_nbrs int64 [nq] optional.  stream: a
        cudaStream_t handle, 0 for the legacy default stream, or None for
        torch's current stream on the engine's GPU.
        """
        import torch
        f32, i32 = torch.float32, torch.int32
        nq = self._queries(d_queries, "d_queries")
        k = params.topk
        args = (self._arg(d_queries, "d_queries", f32), self._arg(d_ids, "d_ids", i32, nq * k),
                self._arg(d_dists, "d_dists", f32, nq * k), self._arg(d_found, "d_found", i32, nq),
                self._arg(d_steps, "d_steps", i32, nq), self._arg(d_nbrs, "d_nbrs", torch.int64, nq))
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        o = params.to_c()
        # 0 is the legacy default stream (cudaStreamLegacy, handle 0x1); a null handle would select the
        # engine's own stream, which is not ordered after torch's work.
        st = C.c_void_p(1 if stream == 0 else stream)
        _check(self._lib.qv_search_device(self._h, args[0], nq, C.byref(o), *args[1:], st))

    def check_device_status(self) -> None:
        _check(self._lib.qv_check_device_status(self._h))

    # component kernels (torch CUDA tensors) -------------------------------
    # The component calls run on the engine's own stream and return when their kernel has finished; torch's
    # current stream is drained first, so inputs that torch kernels produced are complete.
    def _drain_torch(self) -> None:
        import torch
        torch.cuda.current_stream(self.device).synchronize()

    def build_lut(self, d_queries, d_lut, d_q2) -> None:
        """d_queries float32 [nq, dim] -> d_lut float32 [nq, M, 256] and q'' d_q2 float32 [nq, dim]."""
        import torch
        nq = self._queries(d_queries, "d_queries")
        args = (self._arg(d_queries, "d_queries", torch.float32),
                self._arg(d_lut, "d_lut", torch.float32, nq * self._M * 256),
                self._arg(d_q2, "d_q2", torch.float32, nq * self._dim))
        self._drain_torch()
        _check(self._lib.qv_build_lut_device(self._h, args[0], nq, args[1], args[2], None))

    def _pairs(self, d_query_of, d_ids, d_out):
        import torch
        n = d_ids.numel()
        return n, (self._arg(d_query_of, "d_query_of", torch.int32, n), self._arg(d_ids, "d_ids", torch.int32),
                   self._arg(d_out, "d_out", torch.float32, n))

    def adc(self, d_lut, d_query_of, d_ids, d_out) -> None:
        """d_out[i] = ADC of code d_ids[i] under LUT d_lut[d_query_of[i]] (d_lut float32 [nq, M, 256])."""
        import torch
        lut = self._arg(d_lut, "d_lut", torch.float32)
        if d_lut.numel() % (self._M * 256) != 0:
            raise ValueError(f"d_lut must be float32 [nq, {self._M}, 256]")
        n, (qof, ids, out) = self._pairs(d_query_of, d_ids, d_out)
        self._drain_torch()
        _check(self._lib.qv_adc_device(self._h, lut, qof, ids, n, out, None))

    def exact_l2(self, d_q2, d_query_of, d_ids, d_out) -> None:
        """d_out[i] = exact squared L2 of q'' d_q2[d_query_of[i]] (float32 [nq, dim]) and node d_ids[i]."""
        import torch
        self._queries(d_q2, "d_q2")
        q2 = self._arg(d_q2, "d_q2", torch.float32)
        n, (qof, ids, out) = self._pairs(d_query_of, d_ids, d_out)
        self._drain_torch()
        _check(self._lib.qv_exact_l2_device(self._h, q2, qof, ids, n, out, None))


def open_index_arrays(index_dir: str | Path, data_type: str) -> dict:
    """Read an index directory into host arrays (for Engine.from_arrays)."""
    index_dir = Path(index_dir)
    disk = sorted(index_dir.glob("*_disk.index"))
    piv = sorted(index_dir.glob("*_pq_pivots.bin"))
    if len(disk) != 1 or len(piv) != 1:
        raise FileNotFoundError(f"expected one *_disk.index and one *_pq_pivots.bin in {index_dir}")
    lay = formats.read_disk_index_header(disk[0], data_type)
    pq = formats.read_pq(str(piv[0])[: -len("_pq_pivots.bin")])
    return {"layout": lay, "pages": formats.read_pages(disk[0], lay.num_pages), **pq}
