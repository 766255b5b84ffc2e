"""NumPy front end of the Quiver search engine.

Same interface and error behaviour as Quiver's Python API
(python/quiver/index.py in ruc-system/quiver-ae): ``IndexQuiver(index_dir,
...)`` validates its options, and ``search`` writes the queries to a
temporary ``.fbin/.u8bin/.i8bin`` file, runs the ``quiver_search``
executable with the reference's flags, and reads back
``result_ids.bin`` / ``result_distances.bin``.  The executable found by
default is this repository's B200 build (``quiver-ae_b200/bin/quiver_search``).
"""
from __future__ import annotations

import os
import shutil
import struct
import subprocess
import tempfile
from pathlib import Path
from typing import Mapping, Sequence

import numpy as np


class QuiverError(RuntimeError):
    """The engine could not run or did not return valid results."""


# data_type -> (on-disk dtype, query file suffix); the suffix selects the
# element type in load_queries_as_float (bin/common/data_io.hpp:73-108).
_TYPES = {
    "float": (np.dtype("<f4"), ".fbin"),
    "float32": (np.dtype("<f4"), ".fbin"),
    "uint8": (np.dtype("u1"), ".u8bin"),
    "int8": (np.dtype("i1"), ".i8bin"),
}
_PKG_BIN = Path(__file__).resolve().parents[1] / "bin" / "quiver_search"


def _require_positive(value, name: str) -> int:
    v = int(value)
    if v <= 0:
        raise ValueError(f"{name} must be positive")
    return v


class IndexQuiver:
    """Search one index directory; results come back as NumPy arrays."""

    def __init__(
        self,
        index_dir: str | os.PathLike[str],
        *,
        data_type: str = "float32",
        ssds: Sequence[str] | None = None,
        ssd_list_file: str | os.PathLike[str] | None = None,
        spdk_base_lba: int | None = None,
        binary: str | os.PathLike[str] | None = None,
        memory_backend: str = "heap",
        num_blocks: int = 756,
        queries_per_block: int = 1,
        pipe_width: int = 2,
        poll_threads: int = 6,
        runners_per_ssd: int = 1,
        env: Mapping[str, str] | None = None,
    ) -> None:
        self.index_dir = Path(index_dir).expanduser().resolve()
        if not self.index_dir.is_dir():
            raise ValueError(f"index_dir is not a directory: {self.index_dir}")
        kind = data_type.lower()
        if kind not in _TYPES:
            raise ValueError("data_type must be float32, float, uint8, or int8")
        self.data_type = "float" if kind == "float32" else kind
        self._numpy_dtype, self._query_suffix = _TYPES[kind]
        if ssds and ssd_list_file:
            raise ValueError("pass either ssds or ssd_list_file, not both")
        self.ssds = tuple(str(s).strip() for s in (ssds or ()))
        if any(not s for s in self.ssds):
            raise ValueError("SSD PCI addresses must not be empty")
        self.ssd_list_file = Path(ssd_list_file).expanduser().resolve() if ssd_list_file else None
        if self.ssd_list_file and not self.ssd_list_file.is_file():
            raise ValueError(f"ssd_list_file does not exist: {self.ssd_list_file}")
        if spdk_base_lba is not None and spdk_base_lba < 0:
            raise ValueError("spdk_base_lba must be non-negative")
        self.spdk_base_lba = spdk_base_lba
        if memory_backend not in ("heap", "mmap"):
            raise ValueError("memory_backend must be heap or mmap")
        self.memory_backend = memory_backend
        self.binary = self._locate(binary)
        self.num_blocks = _require_positive(num_blocks, "num_blocks")
        self.queries_per_block = _require_positive(queries_per_block, "queries_per_block")
        self.pipe_width = _require_positive(pipe_width, "pipe_width")
        self.poll_threads = _require_positive(poll_threads, "poll_threads")
        self.runners_per_ssd = _require_positive(runners_per_ssd, "runners_per_ssd")
        self.env = dict(env or {})

    @property
    def num_ssds(self) -> int:
        if self.ssds:
            return len(self.ssds)
        if self.ssd_list_file is None:
            return 0
        lines = self.ssd_list_file.read_text().splitlines()
        return sum(1 for ln in lines if ln.strip() and not ln.lstrip().startswith("#"))

    def search(
        self,
        queries,
        topk: int = 10,
        *,
        ef_search: int = 50,
        early_exit_policy: str = "gpruning",
        timeout: float | None = None,
        extra_args: Sequence[str] = (),
    ) -> tuple[np.ndarray, np.ndarray]:
        """Return ``(ids int32, distances float32)``, both ``(len(queries), topk)``."""
        topk = _require_positive(topk, "topk")
        ef_search = _require_positive(ef_search, "ef_search")
        if early_exit_policy not in ("gpruning", "none"):
            raise ValueError("early_exit_policy must be gpruning or none")
        if timeout is not None and timeout <= 0:
            raise ValueError("timeout must be positive")
        q = np.asarray(queries)
        if q.ndim == 1:
            q = q.reshape(1, -1)
        if q.ndim != 2 or q.shape[0] == 0 or q.shape[1] == 0:
            raise ValueError("queries must be a non-empty 1D or 2D array")
        q = np.ascontiguousarray(q, dtype=self._numpy_dtype)

        with tempfile.TemporaryDirectory(prefix="quiver-python-") as tmp:
            work = Path(tmp)
            qfile = work / f"queries{self._query_suffix}"
            prefix = work / "result"
            with qfile.open("wb") as f:
                f.write(struct.pack("<ii", q.shape[0], q.shape[1]))
                f.write(q.tobytes(order="C"))
            argv = [str(self.binary),
                    "--index-dir", str(self.index_dir), "--query", str(qfile),
                    "--data-type", self.data_type, "--topk", str(topk), "--ef-search", str(ef_search),
                    "--repeat", "1", "--num-blocks", str(self.num_blocks),
                    "--queries-per-block", str(self.queries_per_block), "--pipe-width", str(self.pipe_width),
                    "--poll-threads", str(self.poll_threads), "--runners-per-ssd", str(self.runners_per_ssd),
                    "--memory-backend", self.memory_backend, "--early-exit-policy", early_exit_policy,
                    "--result-prefix", str(prefix)]
            ssd_list = self._ssd_list_path(work)
            if ssd_list is not None:
                argv += ["--ssd-list-file", str(ssd_list)]
            argv += [str(a) for a in extra_args]
            env = {**os.environ, **self.env}
            if self.spdk_base_lba is not None:
                env["SPDK_BASE_LBA"] = str(self.spdk_base_lba)
            try:
                proc = subprocess.run(argv, env=env, text=True, capture_output=True, check=False, timeout=timeout)
            except subprocess.TimeoutExpired as err:
                raise QuiverError(f"quiver_search exceeded the {timeout:g} second timeout") from err
            if proc.returncode != 0:
                detail = proc.stderr.strip() or proc.stdout.strip()
                raise QuiverError(f"quiver_search exited with code {proc.returncode}: {detail}")
            ids = self._read_result(work / "result_ids.bin", np.int32)
            dists = self._read_result(work / "result_distances.bin", np.float32)
        want = (q.shape[0], topk)
        if ids.shape != want or dists.shape != want:
            raise QuiverError(f"unexpected result shape: ids={ids.shape}, distances={dists.shape}, expected={want}")
        return ids, dists

    def _ssd_list_path(self, work: Path) -> Path | None:
        if self.ssd_list_file:
            return self.ssd_list_file
        if not self.ssds:
            return None
        path = work / "ssds.txt"
        path.write_text("".join(f"{s}\n" for s in self.ssds), encoding="ascii")
        return path

    @staticmethod
    def _read_result(path: Path, dtype) -> np.ndarray:
        if not path.is_file():
            raise QuiverError(f"quiver_search did not create {path.name}")
        with path.open("rb") as f:
            head = f.read(8)
            if len(head) != 8:
                raise QuiverError(f"invalid result header in {path}")
            n, d = struct.unpack("<ii", head)
            if n < 0 or d < 0:
                raise QuiverError(f"invalid result dimensions in {path}")
            data = np.fromfile(f, dtype=np.dtype(dtype).newbyteorder("<"))
        if data.size != n * d:
            raise QuiverError(f"truncated result data in {path}")
        return data.reshape(n, d)

    @staticmethod
    def _locate(binary) -> Path:
        if binary:
            cands = [Path(binary).expanduser()]
        elif os.environ.get("QUIVER_BINARY"):
            cands = [Path(os.environ["QUIVER_BINARY"]).expanduser()]
        else:
            cands = [Path(p) for p in (shutil.which("quiver_search"),) if p] + [_PKG_BIN]
        for c in cands:
            r = c.resolve()
            if r.is_file() and os.access(r, os.X_OK):
                return r
        searched = ", ".join(str(c) for c in cands) or "PATH"
        raise QuiverError(f"quiver_search executable not found (searched: {searched})")
