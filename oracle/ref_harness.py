"""Build and call oracle/_ref/libref_quiver.so: the reference's own search kernel.

TEST INFRASTRUCTURE ONLY.  The library is compiled from the reference's
sources where they lie (``<reference>/src``, header-only kernel code, no
external libraries) together with ref_harness.cu, which plays the host side
of the reference's page-request protocol.  It exists to generate golden
outputs that pin the oracle (tests/golden/make_ref_golden.py); it needs a
GPU to run and the reference sources only to build.
"""
from __future__ import annotations

import ctypes as C
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_ref" / "libref_quiver.so"


def reference_root() -> Path | None:
    """The reference project's checkout: $QUIVER_REFERENCE, else the ``reference_path`` that the repository's
    BASELINE.json records; None when neither names an existing directory."""
    where = os.environ.get("QUIVER_REFERENCE")
    if not where:
        baseline = HERE.parent / "BASELINE.json"
        if baseline.is_file():
            import json
            where = json.loads(baseline.read_text()).get("reference_path")
    return Path(where) if where and Path(where).is_dir() else None


def build_if_available(force: bool = False) -> Path | None:
    """Compile the harness when the reference sources are on this machine (see reference_root)."""
    root = reference_root()
    kernel = root / "src" / "quiver" / "kernel_core" / "kernel_q1.cuh" if root else None
    if kernel is None or not kernel.exists():
        return LIB if LIB.exists() else None
    reference_src = root / "src"
    src = HERE / "ref_harness.cu"
    if not force and LIB.exists() and LIB.stat().st_mtime >= src.stat().st_mtime:
        return LIB
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    LIB.parent.mkdir(exist_ok=True)
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-Xcompiler", "-fPIC",
           "-shared", "-I", str(reference_src), str(src), "-o", str(LIB)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference harness build failed:\n{res.stderr}")
    return LIB


def available() -> bool:
    return LIB.exists()


def run(ix, queries: np.ndarray, *, topk: int = 10, ef_search: int = 30, early_exit_policy: str = "none",
        gpruning_warmup_steps: int = 10, gpruning_patience: int = 8, num_blocks: int = 64,
        timeout_s: float = 60.0, nav=None) -> dict:
    """Search with the reference kernel at pipe width 1 on an oracle.OracleIndex
    (with its in-kernel nav entry search when `nav`, an oracle.OracleNav, is given)."""
    lib = C.CDLL(str(LIB))
    lib.ref_run_search.restype = C.c_int
    q = np.ascontiguousarray(queries, dtype=np.float32)
    nq = q.shape[0]
    ids = np.empty((nq, topk), np.int32)
    dists = np.empty((nq, topk), np.float32)
    found = np.empty(nq, np.int32)
    steps = np.empty(nq, np.int32)
    dtype = {"uint8": 0, "float": 1, "int8": 2}[ix.data_type]
    pol = {"none": 0, "gpruning": 2}[early_exit_policy]
    i64, i32 = C.c_int64, C.c_int32
    rc = lib.ref_run_search(
        C.c_void_p(ix.pages.ctypes.data), i64(ix.num_pages), i64(ix.node_size), i64(ix.data_size),
        i64(ix.nodes_per_page), i64(ix.dim), i64(ix.max_degree), i64(ix.num_points), i64(ix.medoid), i32(dtype),
        C.c_void_p(ix.codes.ctypes.data), i32(ix.num_chunks), C.c_void_p(ix.pivots_t.ctypes.data),
        C.c_void_p(ix.centroid.ctypes.data), C.c_void_p(ix.chunk_offsets.ctypes.data), C.c_void_p(q.ctypes.data),
        i32(nq), i32(topk), i32(ef_search), i32(pol), i32(gpruning_warmup_steps), i32(gpruning_patience),
        i32(num_blocks), C.c_void_p(ids.ctypes.data), C.c_void_p(dists.ctypes.data), C.c_void_p(found.ctypes.data),
        C.c_void_p(steps.ctypes.data), C.c_double(timeout_s),
        C.c_void_p(nav.data.ctypes.data if nav is not None else None),
        C.c_void_p(nav.graph.ctypes.data if nav is not None else None),
        C.c_void_p(nav.mapping.ctypes.data if nav is not None else None),
        i32(nav.graph.shape[0] if nav is not None else 0), i32(nav.max_m if nav is not None else 0),
        i32(nav.start if nav is not None else 0))
    if rc != 0:
        raise RuntimeError(f"reference harness returned {rc}")
    return {"ids": ids, "dists": dists, "found": found, "steps": steps}
