"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
for p in (REPO / "quiver-ae_b200", REPO):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built engine")


@pytest.fixture(scope="session", autouse=True)
def _native_libs():
    from quiver_b200 import _build
    _build.build_index_lib()
    from oracle import pyoracle
    pyoracle.build()


def _make_index(root: Path, name: str, *, n: int, dim: int, dtype: str, centers: int, sigma: float, R: int,
                L: int, M: int, nq: int, seed: int):
    from quiver_b200 import builder, formats
    d = root / name
    base = builder.synth_mixture(seed, n, dim, centers, sigma, dtype, stream=0)
    queries = builder.synth_mixture(seed, nq, dim, centers, sigma, dtype, stream=1)
    builder.build_index(d, base, R=R, L=L, alpha=1.2, M=M, passes=2, pq_sample=min(n, 20000), seed=seed)
    gt, _ = builder.ground_truth(base, queries, 10)
    formats.write_bin(d / ("queries" + (".u8bin" if dtype == "uint8" else ".fbin")), queries)
    formats.write_bin(d / "gt.ibin", gt)
    return {"dir": d, "dtype": dtype, "base": base, "queries": queries.astype(np.float32), "gt": gt}


@pytest.fixture(scope="session")
def u8_index(tmp_path_factory):
    """Config-0 shaped (128-d uint8, R=64, M=32) at a size the oracle runs in seconds."""
    return _make_index(tmp_path_factory.mktemp("idx"), "u8", n=6000, dim=128, dtype="uint8", centers=12,
                       sigma=20.0, R=64, L=64, M=32, nq=96, seed=11)


@pytest.fixture(scope="session")
def f32_index(tmp_path_factory):
    """Config-1 shaped (96-d unit-norm float32, R=64, M=32)."""
    return _make_index(tmp_path_factory.mktemp("idx"), "f32", n=4000, dim=96, dtype="float", centers=10,
                       sigma=0.1, R=64, L=64, M=32, nq=64, seed=12)


@pytest.fixture(scope="session")
def i8_index(tmp_path_factory):
    """Signed 8-bit vectors (96-d, R=64, M=32), the reference's int8 element type (.i8bin): a seeded
    12-cluster mixture drawn with numpy (the synthetic generator makes uint8 and float only)."""
    from quiver_b200 import builder, formats
    rng = np.random.default_rng(15)
    centers = rng.integers(-100, 100, size=(12, 96))

    def draw(n):
        x = centers[rng.integers(0, 12, n)] + rng.normal(0.0, 18.0, (n, 96))
        return np.clip(np.rint(x), -128, 127).astype(np.int8)

    base, queries = draw(4000), draw(64)
    d = tmp_path_factory.mktemp("idx") / "i8"
    builder.build_index(d, base, R=64, L=64, alpha=1.2, M=32, passes=2, pq_sample=4000, seed=15)
    gt, _ = builder.ground_truth(base, queries, 10)
    formats.write_bin(d / "queries.i8bin", queries)
    formats.write_bin(d / "gt.ibin", gt)
    return {"dir": d, "dtype": "int8", "base": base, "queries": queries.astype(np.float32), "gt": gt}


@pytest.fixture(scope="session")
def odd_index(tmp_path_factory):
    """Uncommon shapes: R=100 (>64 neighbours per node), M=12 (generic code path), dim=48."""
    return _make_index(tmp_path_factory.mktemp("idx"), "odd", n=2500, dim=48, dtype="uint8", centers=6,
                       sigma=25.0, R=100, L=110, M=12, nq=48, seed=13)


def reference_python_root() -> Path:
    """Where the reference's unmodified Python package (``quiver``) is installed: $QUIVER_REFERENCE_PY, else
    baseline/_ref (``__graft_entry__.build()`` installs it there from the reference sources when they are
    present)."""
    import os
    return Path(os.environ.get("QUIVER_REFERENCE_PY", REPO / "baseline" / "_ref"))


@pytest.fixture(scope="session")
def reference_quiver():
    """The reference's own ``quiver`` module, imported unchanged; skips when it is not installed."""
    root = reference_python_root()
    if not (root / "quiver" / "index.py").is_file():
        pytest.skip(f"the reference's Python package is not installed under {root}")
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    import quiver
    assert Path(quiver.__file__).resolve().is_relative_to(root.resolve()), quiver.__file__
    return quiver
