"""IndexQuiver: the reference's Python API contract (python/tests/test_index.py
in ruc-system/quiver-ae) held by this repository's front end, plus the CLI's
argument validation, which runs before any device work."""
from __future__ import annotations

import stat
import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

ENGINE_STUB = r'''#!/usr/bin/env python3
import struct, sys
from pathlib import Path
import numpy as np

argv = sys.argv[1:]
get = lambda flag: argv[argv.index(flag) + 1]
with open(get("--query"), "rb") as f:
    n, d = struct.unpack("<ii", f.read(8))
k = int(get("--topk"))
if "--ssd-list-file" in argv:
    lines = [l for l in Path(get("--ssd-list-file")).read_text().splitlines() if l]
    assert lines == ["0000:01:00.0", "0000:02:00.0"], lines
Path(get("--result-prefix") + ".argv").write_text("\n".join(argv))
for suffix, arr in (("_ids.bin", np.arange(n * k, dtype="<i4")),
                    ("_distances.bin", np.arange(n * k, dtype="<f4") / 10)):
    with open(get("--result-prefix") + suffix, "wb") as f:
        f.write(struct.pack("<ii", n, k) + arr.tobytes())
'''


def _exe(path: Path, text: str) -> Path:
    path.write_text(text)
    path.chmod(path.stat().st_mode | stat.S_IXUSR)
    return path


@pytest.fixture()
def index_dir(tmp_path):
    d = tmp_path / "index"
    d.mkdir()
    return d


def test_results_and_ssd_list(tmp_path, index_dir):
    from quiver import IndexQuiver
    eng = _exe(tmp_path / "quiver_search", ENGINE_STUB)
    idx = IndexQuiver(index_dir, data_type="float32", ssds=["0000:01:00.0", "0000:02:00.0"], binary=eng)
    ids, dists = idx.search(np.ones((3, 4), dtype=np.float64), topk=2)
    assert idx.num_ssds == 2
    assert ids.dtype == np.dtype("<i4") and dists.dtype == np.dtype("<f4")
    np.testing.assert_array_equal(ids, [[0, 1], [2, 3], [4, 5]])
    np.testing.assert_allclose(dists, [[0.0, 0.1], [0.2, 0.3], [0.4, 0.5]])


def test_argv_contract(tmp_path, index_dir, monkeypatch):
    """The flags a caller sees on the engine's command line (index.py:136-169)."""
    from quiver import IndexQuiver
    eng = _exe(tmp_path / "quiver_search", ENGINE_STUB)
    seen = {}
    real_run = subprocess.run

    def spy(cmd, **kw):
        seen["argv"] = cmd
        return real_run(cmd, **kw)

    monkeypatch.setattr(subprocess, "run", spy)
    IndexQuiver(index_dir, data_type="uint8", binary=eng, pipe_width=4, queries_per_block=2).search(
        np.ones((2, 8)), topk=5, ef_search=70, early_exit_policy="none")
    argv = seen["argv"]
    flag = lambda f: argv[argv.index(f) + 1]
    assert flag("--data-type") == "uint8" and flag("--topk") == "5" and flag("--ef-search") == "70"
    assert flag("--repeat") == "1" and flag("--pipe-width") == "4" and flag("--queries-per-block") == "2"
    assert flag("--num-blocks") == "756" and flag("--early-exit-policy") == "none"
    assert flag("--query").endswith(".u8bin") and "--ssd-list-file" not in argv


def test_rejects_conflicting_ssd_configuration(tmp_path, index_dir):
    from quiver import IndexQuiver
    eng = _exe(tmp_path / "quiver_search", ENGINE_STUB)
    lst = tmp_path / "ssds.txt"
    lst.write_text("0000:01:00.0\n")
    with pytest.raises(ValueError, match="either ssds or ssd_list_file"):
        IndexQuiver(index_dir, ssds=["0000:01:00.0"], ssd_list_file=lst, binary=eng)


def test_validation_errors(tmp_path, index_dir):
    from quiver import IndexQuiver
    eng = _exe(tmp_path / "quiver_search", ENGINE_STUB)
    with pytest.raises(ValueError, match="data_type"):
        IndexQuiver(index_dir, data_type="float16", binary=eng)
    with pytest.raises(ValueError, match="pipe_width must be positive"):
        IndexQuiver(index_dir, pipe_width=0, binary=eng)
    idx = IndexQuiver(index_dir, binary=eng)
    with pytest.raises(ValueError, match="early_exit_policy"):
        idx.search(np.ones((1, 4)), early_exit_policy="darth")
    with pytest.raises(ValueError, match="non-empty"):
        idx.search(np.ones((0, 4)))


def test_reports_engine_failure(tmp_path, index_dir):
    from quiver import IndexQuiver, QuiverError
    eng = _exe(tmp_path / "quiver_search", "#!/usr/bin/env sh\necho 'index metadata is invalid' >&2\nexit 7\n")
    with pytest.raises(QuiverError, match="code 7: index metadata is invalid"):
        IndexQuiver(index_dir, binary=eng).search(np.ones((1, 4), dtype=np.float32))


def test_reports_engine_timeout(tmp_path, index_dir):
    from quiver import IndexQuiver, QuiverError
    eng = _exe(tmp_path / "quiver_search", "#!/usr/bin/env python3\nwhile True:\n    pass\n")
    with pytest.raises(QuiverError, match="exceeded the 0.05 second timeout"):
        IndexQuiver(index_dir, binary=eng).search(np.ones((1, 4), dtype=np.float32), timeout=0.05)


def test_missing_result_file(tmp_path, index_dir):
    from quiver import IndexQuiver, QuiverError
    eng = _exe(tmp_path / "quiver_search", "#!/usr/bin/env sh\nexit 0\n")
    with pytest.raises(QuiverError, match="did not create result_ids.bin"):
        IndexQuiver(index_dir, binary=eng).search(np.ones((1, 4), dtype=np.float32))


# ------------------------------------------------ the real quiver_search --

@pytest.fixture(scope="module")
def cli():
    from quiver_b200 import _build
    _build.build_engine()
    return _build.build_cli()


def _run(cli, *args):
    return subprocess.run([str(cli), *map(str, args)], capture_output=True, text=True, timeout=60)


def test_default_binary_is_this_build(index_dir, cli, monkeypatch):
    from quiver import IndexQuiver
    monkeypatch.delenv("QUIVER_BINARY", raising=False)
    monkeypatch.setenv("PATH", "/usr/bin:/bin")
    assert IndexQuiver(index_dir).binary == Path(cli).resolve()


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
