"""qv_search_noalloc: the search for callers that may not allocate device memory.

Some callers cannot call cudaMalloc once their index is loaded -- a plugin
inside a host application that owns the device allocator, or a serving loop
that cannot afford an allocation's implicit synchronisation or its failure
under memory pressure.  For them the search kernel keeps its scratch (work
counter, error words, device copies of queries and results) in a fixed 4 MiB
device array compiled into the library.  This test calls the entry point
through the C ABI twice in a row and checks that it returns exactly what the
allocating entry point qv_search returns, that a batch too large for the
array is refused with an error instead of being run (also a batch so large
that its byte count would overflow), and that the device's free memory is the
same before and after no-alloc calls made right after the engine is opened.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.gpu
def test_noalloc_search_matches_allocating_search():
    from quiver_b200 import Engine, QuiverEngineError, SearchParams, _build, _lib, formats
    _build.build_engine()
    q = formats.read_bin(GOLDEN / "idx_u8" / "queries.fbin", np.float32)
    import torch
    lib = _lib.engine_lib()
    with Engine.open(GOLDEN / "idx_u8", "uint8") as eng:
        # the first no-alloc call after opening places nothing new on the device
        p0 = SearchParams(topk=10, ef_search=45, pipe_width=2, early_exit_policy="none")
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info(0)[0]
        first = [eng.search_noalloc(q, p0) for _ in range(3)]
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info(0)[0] == free0
        for a, b in zip(first[0], first[2]):
            np.testing.assert_array_equal(a, b)
        for params in (SearchParams(topk=10, ef_search=45, pipe_width=2, early_exit_policy="none"),
                       SearchParams(topk=16, ef_search=30, pipe_width=1, early_exit_policy="gpruning")):
            ref = eng.search(q, params)
            for _ in range(2):  # the scratch array keeps the previous call's contents
                got = eng.search_noalloc(q, params)
                for a, b in zip(got, ref):
                    np.testing.assert_array_equal(a, b)
        # raw C ABI call with a batch above the scratch maximum: refused, nothing launched
        big = 8000
        qb = np.zeros((big, q.shape[1]), np.float32)
        ids = np.empty((big, 10), np.int32)
        dists = np.empty((big, 10), np.float32)
        o = SearchParams(topk=10, ef_search=45).to_c()
        rc = lib.qv_search_noalloc(eng._h, C.c_void_p(qb.ctypes.data), big, q.shape[1], C.byref(o),
                                   C.c_void_p(ids.ctypes.data), C.c_void_p(dists.ctypes.data), None)
        assert rc == _lib.QV_OK + 1  # QV_ERR_INVALID_ARG
        assert "above its 4194304-byte maximum" in lib.qv_last_error().decode()
        # a count whose byte sizes would wrap around 64 bits: refused before any copy
        rc = lib.qv_search_noalloc(eng._h, C.c_void_p(qb.ctypes.data), 1 << 60, q.shape[1], C.byref(o),
                                   C.c_void_p(ids.ctypes.data), C.c_void_p(dists.ctypes.data), None)
        assert rc == _lib.QV_OK + 1
        assert "above its 4194304-byte maximum" in lib.qv_last_error().decode()
        # the engine still works after the refusal
        again = eng.search_noalloc(q, SearchParams(topk=10, ef_search=45, pipe_width=2,
                                                   early_exit_policy="none"))
        np.testing.assert_array_equal(again[0], eng.search(q, SearchParams(topk=10, ef_search=45, pipe_width=2,
                                                                            early_exit_policy="none"))[0])
