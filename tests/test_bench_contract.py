"""bench.py's JSON-line contract, checked through its reference arm (the oracle on the host cores), which
needs no GPU: one line with the required keys, the reference arm's own cpu_baseline and zero-byte e2e,
warm-up raised to 3, and silent non-zero ranks under torchrun."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def _bench(tmp_path, *args, env_extra=None):
    env = dict(os.environ, QUIVER_B200_CACHE=str(tmp_path / "cache"))
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(REPO / "bench.py"), *args], capture_output=True, text=True,
                          env=env, cwd=tmp_path, timeout=600)


def test_reference_arm_prints_one_contract_line(tmp_path):
    res = _bench(tmp_path, "--impl", "reference", "--config", "config0-20k", "--steps", "2", "--warmup", "1")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 2, 3)
    assert line["unit"] == "queries/s" and line["higher_is_better"] is True and line["value"] > 0
    per_step = line["value"] * line["ms_per_step"] / 1000.0  # queries in one step
    assert 64 <= round(per_step) <= 2000 and abs(per_step - round(per_step)) < 1e-6 * per_step
    assert line["config"]["workload"].startswith("config0-20k")
    assert line["config"]["recall_at_10"] >= 0.90
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == line["value"] and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "queries/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work(tmp_path):
    res = _bench(tmp_path, "--impl", "reference", "--config", "config0-20k", "--steps", "1",
                 env_extra={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ""
    assert not (tmp_path / "cache").exists()  # no index built on a rank that does no work
