"""The Python search API.

* ``quiver_b200.IndexQuiver``, the in-process front end: the reference's
  constructor and ``search`` arguments (python/quiver/index.py:27-116), with
  the same ``ValueError`` messages as the reference's module for every bad
  argument, checked side by side against that module, unchanged, when it is
  installed (baseline/_ref or $QUIVER_REFERENCE_PY).
* The reference's module itself finds this repository's CLI through
  ``QUIVER_BINARY`` (index.py:244-264).
* The CLI's argument validation, which runs before any device work.
"""
from __future__ import annotations

import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest


@pytest.fixture()
def index_dir(tmp_path):
    d = tmp_path / "index"
    d.mkdir()
    return d


# (constructor kwargs, search kwargs or None) -> each raises ValueError in both front ends
BAD_ARGUMENTS = [
    ({"data_type": "float16"}, None),
    ({"pipe_width": 0}, None),
    ({"num_blocks": -3}, None),
    ({"queries_per_block": 0}, None),
    ({"poll_threads": 0}, None),
    ({"runners_per_ssd": 0}, None),
    ({"memory_backend": "disk"}, None),
    ({"ssds": ["0000:01:00.0", " "]}, None),
    ({"spdk_base_lba": -1}, None),
    ({"ssd_list_file": "/nonexistent/ssds.txt"}, None),
    ({}, {"topk": 0}),
    ({}, {"ef_search": -1}),
    ({}, {"early_exit_policy": "darth"}),
    ({}, {"timeout": 0}),
    ({}, {"queries": np.ones((0, 4))}),
    ({}, {"queries": np.ones((2, 2, 2))}),
]


def _error_of(cls, index_dir, ctor, search, binary):
    try:
        extra = {"binary": binary} if binary is not None else {}
        idx = cls(index_dir, **ctor, **extra)
        if search is not None:
            kw = dict(search)
            q = kw.pop("queries", np.ones((1, 4), np.float32))
            idx.search(q, **kw)
    except ValueError as err:
        return str(err)
    return None


@pytest.mark.parametrize("ctor,search", BAD_ARGUMENTS)
def test_front_end_refuses_bad_arguments(index_dir, ctor, search):
    from quiver_b200 import IndexQuiver
    assert _error_of(IndexQuiver, index_dir, ctor, search, None) is not None


@pytest.mark.parametrize("ctor,search", BAD_ARGUMENTS)
def test_front_end_messages_match_the_reference_module(reference_quiver, index_dir, tmp_path, ctor, search):
    """Same ValueError text as the reference's unmodified module for the same bad argument (the reference
    needs an executable to construct; a stub that is never run stands in)."""
    from quiver_b200 import IndexQuiver
    stub = tmp_path / "quiver_search"
    stub.write_text("#!/bin/sh\nexit 3\n")
    stub.chmod(0o755)
    want = _error_of(reference_quiver.IndexQuiver, index_dir, ctor, search, stub)
    got = _error_of(IndexQuiver, index_dir, ctor, search, None)
    assert want is not None
    assert got == want


def test_front_end_directory_and_ssd_conflict(index_dir, tmp_path):
    from quiver_b200 import IndexQuiver
    with pytest.raises(ValueError, match="index_dir is not a directory"):
        IndexQuiver(tmp_path / "missing")
    lst = tmp_path / "ssds.txt"
    lst.write_text("0000:01:00.0\n# comment\n\n0000:02:00.0\n")
    with pytest.raises(ValueError, match="either ssds or ssd_list_file"):
        IndexQuiver(index_dir, ssds=["0000:01:00.0"], ssd_list_file=lst)
    assert IndexQuiver(index_dir, ssd_list_file=lst).num_ssds == 2
    assert IndexQuiver(index_dir, ssds=["a", "b", "c"]).num_ssds == 3


def test_front_end_refuses_ssds_and_unknown_flags_before_loading(index_dir):
    """No SPDK here: a search with SSDs configured fails as in a build without SPDK, before the index is
    opened; CLI flags the in-process engine does not take are refused the same way."""
    from quiver_b200 import IndexQuiver, QuiverError
    with pytest.raises(QuiverError, match="without SPDK support"):
        IndexQuiver(index_dir, ssds=["0000:01:00.0"]).search(np.ones((1, 4), np.float32))
    idx = IndexQuiver(index_dir)
    with pytest.raises(QuiverError, match="not supported by the in-process engine"):
        idx.search(np.ones((1, 4), np.float32), extra_args=["--per-step-recall"])
    assert idx._engine is None


def test_reference_module_finds_this_cli(reference_quiver, index_dir, monkeypatch):
    """The reference's module, unchanged, resolves QUIVER_BINARY to this repository's CLI."""
    from quiver_b200 import _build
    cli = _build.build_cli()
    monkeypatch.setenv("QUIVER_BINARY", str(cli))
    assert reference_quiver.IndexQuiver(index_dir).binary == Path(cli).resolve()


# ------------------------------------------------ the real quiver_search --

@pytest.fixture(scope="module")
def cli():
    from quiver_b200 import _build
    _build.build_engine()
    return _build.build_cli()


def _run(cli, *args):
    return subprocess.run([str(cli), *map(str, args)], capture_output=True, text=True, timeout=60)


@pytest.mark.parametrize("args,msg", [
    (["--pipe-width", "17"], "--pipe-width must be in [1, 16]"),
    (["--queries-per-block", "9"], "--queries-per-block must be in [1, 8]"),
    (["--num-blocks", "0"], "--num-blocks must be positive"),
    (["--early-exit-policy", "darth"], "invalid --early-exit-policy"),
    (["--memory-backend", "disk"], "Unsupported --memory-backend"),
])
def test_cli_validation(cli, index_dir, tmp_path, args, msg):
    q = tmp_path / "q.fbin"
    q.write_bytes(struct.pack("<ii", 1, 4) + np.ones(4, np.float32).tobytes())
    r = _run(cli, "--index-dir", index_dir, "--query", q, "--data-type", "float", *args)
    assert r.returncode == 1
    assert msg in r.stderr


def test_cli_required_flags_and_spdk(cli, index_dir, tmp_path):
    r = _run(cli, "--query", "x.fbin", "--data-type", "float")
    assert r.returncode == 1 and "--index-dir" in r.stderr
    lst = tmp_path / "ssds.txt"
    lst.write_text("0000:01:00.0\n")
    r = _run(cli, "--index-dir", index_dir, "--query", "x.fbin", "--data-type", "float", "--ssd-list-file", lst)
    assert r.returncode == 1 and "without SPDK support" in r.stderr


def test_cli_reports_missing_index(cli, index_dir, tmp_path):
    q = tmp_path / "q.fbin"
    q.write_bytes(struct.pack("<ii", 1, 4) + np.ones(4, np.float32).tobytes())
    r = _run(cli, "--index-dir", index_dir, "--query", q, "--data-type", "float")
    assert r.returncode == 1 and "No *_disk.index or disk.index found" in r.stderr


def _bare_engine(device=0, dim=8, M=2):
    """An Engine object with no library handle: only the Python-side argument checks can run on it."""
    from quiver_b200 import Engine
    e = Engine.__new__(Engine)
    e._h, e.device, e._dim, e._M = None, device, dim, M
    return e


def test_tensor_methods_refuse_bad_tensors_before_any_device_call():
    import torch
    from quiver_b200 import SearchParams
    e = _bare_engine()
    p = SearchParams(topk=3)
    cpu_q = torch.zeros((5, 8), dtype=torch.float32)
    with pytest.raises(ValueError, match="CUDA tensor on cuda:0"):
        e.search_device(cpu_q, p, torch.zeros((5, 3), dtype=torch.int32), torch.zeros((5, 3)))
    with pytest.raises(ValueError, match=r"\[nq, 8\]"):
        e.search_device(torch.zeros((5, 7)), p, None, None)
    with pytest.raises(ValueError, match=r"\[nq, 8\]"):
        e.build_lut(torch.zeros(40), None, None)
    with pytest.raises(ValueError, match=r"\[nq, 8\]"):
        e.search_device(np.zeros((5, 8), np.float32), p, None, None)  # a host array, not a tensor
    with pytest.raises(ValueError, match="CUDA tensor"):
        e.exact_l2(cpu_q, torch.zeros(4, dtype=torch.int32), torch.zeros(4, dtype=torch.int32), torch.zeros(4))
    with pytest.raises(ValueError, match="CUDA tensor"):
        e.adc(torch.zeros((5, 2, 256)), torch.zeros(4, dtype=torch.int32), torch.zeros(4, dtype=torch.int32),
              torch.zeros(4))


def test_tensor_argument_check_messages():
    """dtype, contiguity and size are checked in that order once the tensor is on the engine's GPU; on a
    host without a GPU the device check comes first."""
    import torch
    e = _bare_engine()
    t = torch.zeros(6, dtype=torch.float32)
    assert e._arg(None, "x", torch.float32) is None
    with pytest.raises(ValueError, match="x must be a CUDA tensor on cuda:0"):
        e._arg(t, "x", torch.float32, 6)
    with pytest.raises(ValueError, match="must be a CUDA tensor"):
        e._arg(t.numpy(), "x", torch.float32)


def test_adc_batch_refuses_host_tensors():
    import torch
    from quiver_b200.adc import adc_batch
    with pytest.raises(ValueError, match="codes must be a CUDA uint8"):
        adc_batch(torch.zeros((10, 32), dtype=torch.uint8), torch.zeros((1, 32, 256)),
                  torch.zeros((1, 4), dtype=torch.int32))
