"""ctypes view of the C ABIs in include/quiver_b200.h and include/quiver_b200_build.h.

The engine library is the only search path: if it is missing, loading fails
with an error instead of falling back to any host implementation.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

from . import _build

QV_OK = 0
(QV_ERR_INVALID_ARG, QV_ERR_IO, QV_ERR_BAD_INDEX, QV_ERR_CUDA, QV_ERR_DEVICE, QV_ERR_UNSUPPORTED,
 QV_ERR_OOM) = range(1, 8)
QV_UINT8, QV_FLOAT, QV_INT8 = 0, 1, 2
QV_PAGES_HBM, QV_PAGES_HOST, QV_PAGES_STRIPED, QV_PAGES_SHARED = 0, 1, 2, 3
QV_STRIPE_HANDLE_BYTES = 64
QV_NOALLOC_SCRATCH_BYTES = 4 << 20
QV_EXIT_NONE, QV_EXIT_GPRUNING = 0, 2
QV_LUT_FP32 = 0
QV_ADC_AUTO, QV_ADC_THREAD, QV_ADC_PIPE = 0, 1, 2

DTYPE_CODES = {"uint8": QV_UINT8, "float": QV_FLOAT, "float32": QV_FLOAT, "int8": QV_INT8}


class NativeLibraryMissing(RuntimeError):
    """Raised when a compiled quiver_b200 library has not been built."""


class IndexInfo(C.Structure):
    _fields_ = [
        ("num_points", C.c_int64), ("dim", C.c_int64), ("max_degree", C.c_int64),
        ("node_size", C.c_int64), ("data_size", C.c_int64), ("nodes_per_page", C.c_int64),
        ("num_pages", C.c_int64), ("medoid", C.c_int64), ("data_type", C.c_int32),
        ("num_chunks", C.c_int32),
    ]


class EngineOpts(C.Structure):
    _fields_ = [
        ("index_dir", C.c_char_p), ("data_type", C.c_int32), ("memory_backend", C.c_char_p),
        ("memory_index_file", C.c_char_p), ("device", C.c_int32), ("page_store", C.c_int32),
        ("validate", C.c_int32), ("num_stripes", C.c_int32), ("stripe_devices", C.c_void_p),
        ("stripe_rank", C.c_int32),
    ]


class IndexArrays(C.Structure):
    _fields_ = [
        ("info", IndexInfo), ("pages", C.c_void_p), ("codes", C.c_void_p), ("pivots", C.c_void_p),
        ("centroid", C.c_void_p), ("chunk_offsets", C.c_void_p),
    ]


class SearchOpts(C.Structure):
    _fields_ = [
        ("topk", C.c_int32), ("ef_search", C.c_int32), ("pipe_width", C.c_int32),
        ("queries_per_block", C.c_int32), ("num_blocks", C.c_int32),
        ("early_exit_policy", C.c_int32), ("gpruning_warmup_steps", C.c_int32),
        ("gpruning_patience", C.c_int32), ("lut_mode", C.c_int32), ("skip_nav", C.c_int32),
        ("visited_filter", C.c_int32),
    ]


class SearchStats(C.Structure):
    _fields_ = [
        ("h2d_ms", C.c_double), ("kernel_ms", C.c_double), ("d2h_ms", C.c_double),
        ("total_ms", C.c_double), ("expansions", C.c_int64), ("neighbors_scored", C.c_int64),
        ("grid", C.c_int32), ("slots_per_block", C.c_int32), ("smem_per_block", C.c_int32),
        ("blocks_per_sm", C.c_int32),
    ]


class StreamOpts(C.Structure):
    _fields_ = [("prefeed", C.c_int32), ("admit_min_batch", C.c_int32), ("feed_timeout_ms", C.c_int32),
                ("admit_limit", C.c_int32)]


class StreamStats(C.Structure):
    _fields_ = [
        ("search_ms", C.c_double), ("qps", C.c_double), ("lat_avg_ms", C.c_double), ("lat_p50_ms", C.c_double),
        ("lat_p90_ms", C.c_double), ("lat_p99_ms", C.c_double), ("lat_p999_ms", C.c_double),
        ("lat_max_ms", C.c_double), ("admissions", C.c_int64), ("workers", C.c_int32), ("max_inflight", C.c_int32),
        ("expansions", C.c_int64),
    ]


# Every symbol include/quiver_b200.h declares, with (restype, argtypes).
ENGINE_SYMBOLS = {
    "qv_version": (C.c_char_p, []),
    "qv_last_error": (C.c_char_p, []),
    "qv_search_opts_default": (None, [C.POINTER(SearchOpts)]),
    "qv_index_probe": (C.c_int, [C.c_char_p, C.c_int32, C.POINTER(IndexInfo)]),
    "qv_engine_create": (C.c_int, [C.POINTER(EngineOpts), C.POINTER(C.c_void_p)]),
    "qv_engine_create_from_arrays": (C.c_int, [C.POINTER(IndexArrays), C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    "qv_engine_info": (C.c_int, [C.c_void_p, C.POINTER(IndexInfo)]),
    "qv_engine_set_nav": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32,
                                    C.c_int32]),
    "qv_engine_nav_info": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                     C.POINTER(C.c_int32)]),
    "qv_engine_destroy": (None, [C.c_void_p]),
    "qv_engine_stripe_handle": (C.c_int, [C.c_void_p, C.c_void_p]),
    "qv_engine_attach_stripes": (C.c_int, [C.c_void_p, C.c_void_p]),
    "qv_search": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.POINTER(SearchOpts),
                            C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(SearchStats)]),
    "qv_search_timed": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.POINTER(SearchOpts),
                                  C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(SearchStats)]),
    "qv_stream_opts_default": (None, [C.POINTER(StreamOpts)]),
    "qv_search_stream": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.POINTER(SearchOpts),
                                   C.POINTER(StreamOpts), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.POINTER(StreamStats)]),
    "qv_search_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.POINTER(SearchOpts), C.c_void_p,
                                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "qv_search_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.POINTER(SearchOpts),
                                    C.c_void_p, C.c_void_p, C.c_void_p]),
    "qv_check_device_status": (C.c_int, [C.c_void_p]),
    "qv_plan": (C.c_int, [C.c_void_p, C.POINTER(SearchOpts), C.c_int64, C.POINTER(SearchStats)]),
    "qv_build_lut_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]),
    "qv_adc_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "qv_exact_l2_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p,
                                     C.c_void_p]),
    "qv_synth_mixture_gpu": (C.c_int, [C.c_uint64, C.c_int32, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                       C.c_double, C.c_int32, C.c_void_p, C.c_int32]),
    "qv_pq_encode_gpu": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                   C.c_void_p, C.c_int32, C.c_void_p]),
    "qv_vamana_gpu": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_float,
                                C.c_int32, C.c_uint64, C.c_int32, C.c_void_p, C.c_void_p, C.POINTER(C.c_int64)]),
    "qv_adc_batch": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                               C.c_int64, C.c_void_p, C.c_int32, C.c_void_p]),
}

INDEX_SYMBOLS = {
    "qvb_last_error": (C.c_char_p, []),
    "qvb_synth_mixture": (C.c_int, [C.c_uint64, C.c_int32, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                    C.c_double, C.c_int32, C.c_void_p, C.c_int32]),
    "qvb_ground_truth": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int64, C.c_int32,
                                   C.c_int32, C.c_void_p, C.c_void_p, C.c_int32]),
    "qvb_vamana": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_float,
                             C.c_int32, C.c_uint64, C.c_int32, C.c_void_p, C.c_void_p,
                             C.POINTER(C.c_int64)]),
    "qvb_pq_train": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_int64, C.c_int32,
                               C.c_uint64, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "qvb_pq_encode": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p]),
}

_cache: dict[str, C.CDLL] = {}


def _load(path: Path, symbols: dict) -> C.CDLL:
    key = str(path)
    if key in _cache:
        return _cache[key]
    if not path.exists():
        raise NativeLibraryMissing(
            f"{path.name} is not built; run __graft_entry__.build() or "
            f"python quiver-ae_b200/quiver_b200/_build.py")
    lib = C.CDLL(str(path))
    for name, (res, args) in symbols.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _cache[key] = lib
    return lib


def engine_lib() -> C.CDLL:
    return _load(_build.ENGINE_LIB, ENGINE_SYMBOLS)


def index_lib() -> C.CDLL:
    return _load(_build.INDEX_LIB, INDEX_SYMBOLS)
