"""In-process search front end with the reference's Python signature.

The reference's ``quiver.IndexQuiver`` (python/quiver/index.py:27-203)
writes the queries to a temporary file, runs a new ``quiver_search`` process
for every call -- which loads the whole index again -- and reads the result
files back.  That module keeps working unchanged against this repository's
CLI (set ``QUIVER_BINARY`` or pass ``binary=``).  This class is the
in-process alternative for callers who can link the engine: it accepts the
same constructor and ``search`` arguments, refuses bad ones with the same
``ValueError`` messages, and reports engine failures as ``QuiverError``,
but it opens the index on the GPU once, at the first search, keeps it
resident, and calls the C ABI (``qv_search``) with the caller's arrays
directly -- no files, no process, no reload.

Arguments that only mean something to the reference's SPDK backend
(``ssds``, ``ssd_list_file``, ``spdk_base_lba``, ``poll_threads``,
``runners_per_ssd``) are validated as the reference validates them; a
search with SSDs configured fails as in a build without SPDK.  ``binary``
and ``env`` are accepted and unused: no process is started.  ``timeout``
cannot interrupt a kernel: a search that ran longer raises the reference's
timeout error after it returns.
"""
from __future__ import annotations

import os
import time
from pathlib import Path
from typing import Mapping, Sequence

import numpy as np

from .engine import Engine, QuiverEngineError, SearchParams


class QuiverError(RuntimeError):
    """The engine could not run the search or return valid results."""


# data_type spellings the reference accepts -> (engine type name, element dtype of the query rows)
_TYPE_NAMES = {"float32": ("float", np.float32), "float": ("float", np.float32), "uint8": ("uint8", np.uint8),
               "int8": ("int8", np.int8)}

# CLI flags a caller may pass through extra_args and the search option each one sets
_EXTRA_INT_FLAGS = {"--gpruning-warmup-steps": "gpruning_warmup_steps", "--gpruning-patience": "gpruning_patience"}


def _count(value, name: str) -> int:
    v = int(value)
    if v <= 0:
        raise ValueError(f"{name} must be positive")
    return v


class IndexQuiver:
    """A Quiver index searched on a B200 in this process (see the module docstring).

    Extra keyword arguments over the reference's: ``device`` (CUDA ordinal) and
    ``page_store`` ("hbm" or "host": node records in the GPU's HBM or in pinned
    host DRAM read over PCIe)."""

    def __init__(self, index_dir: str | os.PathLike[str], *, data_type: str = "float32",
                 ssds: Sequence[str] | None = None, ssd_list_file: str | os.PathLike[str] | None = None,
                 spdk_base_lba: int | None = None, binary: str | os.PathLike[str] | None = None,
                 memory_backend: str = "heap", num_blocks: int = 756, queries_per_block: int = 1,
                 pipe_width: int = 2, poll_threads: int = 6, runners_per_ssd: int = 1,
                 env: Mapping[str, str] | None = None, device: int = 0, page_store: str = "hbm") -> None:
        path = Path(index_dir).expanduser().resolve()
        if not path.is_dir():
            raise ValueError(f"index_dir is not a directory: {path}")
        self.index_dir = path
        key = data_type.lower()
        if key not in _TYPE_NAMES:
            raise ValueError("data_type must be float32, float, uint8, or int8")
        self.data_type, self._row_dtype = _TYPE_NAMES[key]
        if ssds and ssd_list_file:
            raise ValueError("pass either ssds or ssd_list_file, not both")
        self.ssds = tuple(str(s).strip() for s in ssds or ())
        if "" in self.ssds:
            raise ValueError("SSD PCI addresses must not be empty")
        self.ssd_list_file = Path(ssd_list_file).expanduser().resolve() if ssd_list_file else None
        if self.ssd_list_file is not None and not self.ssd_list_file.is_file():
            raise ValueError(f"ssd_list_file does not exist: {self.ssd_list_file}")
        if spdk_base_lba is not None and spdk_base_lba < 0:
            raise ValueError("spdk_base_lba must be non-negative")
        self.spdk_base_lba = spdk_base_lba
        if memory_backend not in ("heap", "mmap"):
            raise ValueError("memory_backend must be heap or mmap")
        self.memory_backend = memory_backend
        self.binary = binary
        self.num_blocks = _count(num_blocks, "num_blocks")
        self.queries_per_block = _count(queries_per_block, "queries_per_block")
        self.pipe_width = _count(pipe_width, "pipe_width")
        self.poll_threads = _count(poll_threads, "poll_threads")
        self.runners_per_ssd = _count(runners_per_ssd, "runners_per_ssd")
        self.env = dict(env or {})
        if page_store not in ("hbm", "host"):
            raise ValueError("page_store must be hbm or host")
        self.device = int(device)
        self.page_store = page_store
        self._engine: Engine | None = None

    @property
    def num_ssds(self) -> int:
        if self.ssds:
            return len(self.ssds)
        if self.ssd_list_file is None:
            return 0
        return sum(1 for ln in self.ssd_list_file.read_text().splitlines()
                   if ln.strip() and not ln.lstrip().startswith("#"))

    def _open(self) -> Engine:
        if self._engine is None:
            if self.num_ssds:
                raise QuiverError("SSD page backends need SPDK; this engine was built without SPDK support "
                                  "(pages are served from GPU or host memory)")
            try:
                self._engine = Engine.open(self.index_dir, self.data_type, memory_backend=self.memory_backend,
                                           device=self.device, page_store=self.page_store)
            except QuiverEngineError as err:
                raise QuiverError(f"could not load the index: {err}") from err
        return self._engine

    def _options(self, extra_args: Sequence[str]) -> dict:
        opts: dict = {}
        args = [str(a) for a in extra_args]
        i = 0
        while i < len(args):
            flag = args[i]
            if flag == "--skip-nav":
                opts["skip_nav"] = True
                i += 1
            elif flag in _EXTRA_INT_FLAGS and i + 1 < len(args):
                opts[_EXTRA_INT_FLAGS[flag]] = int(args[i + 1])
                i += 2
            else:
                raise QuiverError(f"extra argument {flag!r} is not supported by the in-process engine "
                                  f"(supported: --skip-nav, {', '.join(_EXTRA_INT_FLAGS)})")
        return opts

    def search(self, queries, topk: int = 10, *, ef_search: int = 50, early_exit_policy: str = "gpruning",
               timeout: float | None = None, extra_args: Sequence[str] = ()) -> tuple[np.ndarray, np.ndarray]:
        """Return ``(ids, distances)``, int32 and float32 arrays of shape ``(len(queries), topk)``; ids are
        -1 and distances +inf where fewer than topk nodes were found, distances are squared L2."""
        topk = _count(topk, "topk")
        ef_search = _count(ef_search, "ef_search")
        if early_exit_policy not in ("gpruning", "none"):
            raise ValueError("early_exit_policy must be gpruning or none")
        if timeout is not None and timeout <= 0:
            raise ValueError("timeout must be positive")
        rows = np.asarray(queries)
        if rows.ndim == 1:
            rows = rows[None, :]
        if rows.ndim != 2 or 0 in rows.shape:
            raise ValueError("queries must be a non-empty 1D or 2D array")
        # the reference hands the engine rows of the index's type, which the CLI widens to float32
        rows = np.ascontiguousarray(rows, dtype=self._row_dtype).astype(np.float32)
        params = SearchParams(topk=topk, ef_search=ef_search, pipe_width=self.pipe_width,
                              queries_per_block=self.queries_per_block, num_blocks=self.num_blocks,
                              early_exit_policy=early_exit_policy, **self._options(extra_args))
        engine = self._open()
        t0 = time.monotonic()
        try:
            ids, dists, _ = engine.search(rows, params)
        except QuiverEngineError as err:
            raise QuiverError(f"search failed: {err}") from err
        if timeout is not None and time.monotonic() - t0 > timeout:
            raise QuiverError(f"quiver_search exceeded the {timeout:g} second timeout")
        return ids, dists

    def close(self) -> None:
        """Release the GPU copy of the index (the next search loads it again)."""
        if self._engine is not None:
            self._engine.close()
            self._engine = None

    def __enter__(self) -> "IndexQuiver":
        return self

    def __exit__(self, *exc) -> None:
        self.close()
