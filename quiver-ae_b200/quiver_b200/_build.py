"""Build recipe for the native parts of quiver_b200.

Everything is compiled in-tree so the shared objects travel with the source:

* ``lib/libquiver_b200.so`` -- the search engine and its C ABI
  (``include/quiver_b200.h``), CUDA for sm_100a only;
* ``lib/libqv_index.so`` -- host index construction and synthetic inputs
  (``include/quiver_b200_build.h``);
* ``bin/quiver_search`` -- the drop-in command-line engine that Quiver's
  Python API (``IndexQuiver``) shells out to.

Objects are rebuilt when a source or header is newer than the target.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]          # quiver-ae_b200/
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
CLI = PKG_ROOT / "cli"
LIB_DIR = PKG_ROOT / "lib"
BIN_DIR = PKG_ROOT / "bin"
OBJ_DIR = PKG_ROOT / "_build"
INCLUDE = REPO_ROOT / "include"

ENGINE_LIB = LIB_DIR / "libquiver_b200.so"
INDEX_LIB = LIB_DIR / "libqv_index.so"
CLI_BIN = BIN_DIR / "quiver_search"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
]
HOST_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-ffp-contract=off", "-mavx2", "-mfma"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return str(cand)
    raise RuntimeError("nvcc not found: the quiver_b200 engine needs the CUDA toolkit to build")


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def _run(cmd: list[str]) -> None:
    res = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(map(str, cmd))}\n{res.stdout}\n{res.stderr}")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def build_engine(force: bool = False, verbose: bool = False) -> Path:
    """Compile libquiver_b200.so (sm_100a)."""
    units = ["engine.cu", "search_u8.cu", "search_i8.cu", "search_f32.cu", "adc_batch.cu", "vamana_gpu.cu", "build_gpu.cu", "index_io.cpp"]
    headers = _headers()
    if not force and ENGINE_LIB.exists() and not _newer(ENGINE_LIB, [CSRC / u for u in units] + headers):
        return ENGINE_LIB
    LIB_DIR.mkdir(exist_ok=True)
    OBJ_DIR.mkdir(exist_ok=True)
    nvcc = _nvcc()
    jobs = []
    objs = []
    for u in units:
        src = CSRC / u
        obj = OBJ_DIR / (u + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + headers):
            if u.endswith(".cu"):
                cmd = [nvcc, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
            else:
                cmd = ["g++", *HOST_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
            jobs.append(cmd)
    if jobs:
        with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
            for f in [ex.submit(_run, j) for j in jobs]:
                f.result()
    if force or jobs or _newer(ENGINE_LIB, objs):
        _run([nvcc, *NVCC_FLAGS, "-shared", *objs, "-o", ENGINE_LIB])
    return ENGINE_LIB


def build_index_lib(force: bool = False) -> Path:
    """Compile libqv_index.so (host, OpenMP)."""
    LIB_DIR.mkdir(exist_ok=True)
    src = CSRC / "index_build.cpp"
    if force or _newer(INDEX_LIB, [src] + _headers()):
        _run(["g++", *HOST_FLAGS, "-fopenmp", "-shared", "-I", INCLUDE, "-I", CSRC, src, "-o", INDEX_LIB])
    return INDEX_LIB


def build_cli(force: bool = False) -> Path:
    """Compile bin/quiver_search against libquiver_b200.so."""
    BIN_DIR.mkdir(exist_ok=True)
    src = CLI / "quiver_search.cpp"
    if not src.exists():
        return CLI_BIN
    if force or _newer(CLI_BIN, [src, ENGINE_LIB] + _headers()):
        _run(["g++", "-O2", "-std=c++17", "-I", INCLUDE, src, "-o", CLI_BIN,
              "-L", LIB_DIR, "-lquiver_b200", f"-Wl,-rpath,$ORIGIN/../lib"])
    return CLI_BIN


def build_all(force: bool = False) -> None:
    build_index_lib(force)
    build_engine(force)
    build_cli(force)


if __name__ == "__main__":
    import sys
    build_all(force="--force" in sys.argv)
    print(ENGINE_LIB, INDEX_LIB, CLI_BIN)
