"""Generate the golden vectors in this directory.

Step 1 (any host, once): ``python tests/golden/make_ref_golden.py index``
builds the two fixture indexes committed here (idx_u8: 128-d uint8, R=64,
M=32, the config-0 shape at N=2000; idx_f32: 96-d unit float32, R=64, M=32,
the config-1 shape at N=1000) and their query files.

Step 2 (a B200 box, reference harness built from the reference sources):
``python tests/golden/make_ref_golden.py ref OUT_DIR`` runs the reference's
own persistent kernel (oracle/_ref, pipe width 1) on both fixtures for every
setting in SETTINGS and writes ``ref_<index>.npz`` into OUT_DIR; the files are
then committed next to this script.

Nav graphs: ``python tests/golden/make_ref_golden.py nav`` builds a nav
graph for each fixture (quiver_b200.builder.build_nav, NAV_SIZES nodes) into
``nav_<index>`` (kept apart from the index directory, which the engine and
the reference would otherwise pick up); ``... refnav OUT_DIR`` runs the
reference kernel with its in-kernel nav entry search on them for every
setting in NAV_SETTINGS and writes ``ref_nav_<index>.npz``.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT / "quiver-ae_b200"), str(ROOT)]

FIXTURES = {
    "idx_u8": dict(n=2000, dim=128, dtype="uint8", centers=20, sigma=20.0, R=64, L=100, M=32, nq=64, seed=101),
    "idx_f32": dict(n=1000, dim=96, dtype="float", centers=10, sigma=0.1, R=64, L=100, M=32, nq=48, seed=102),
}
# (topk, ef_search, early_exit_policy)
SETTINGS = [(10, 10, "none"), (10, 30, "none"), (10, 64, "none"), (10, 45, "gpruning"), (40, 50, "none"),
            (1, 16, "none")]


NAV_SIZES = {"idx_u8": 200, "idx_f32": 120}
NAV_SETTINGS = [(10, 10, "none"), (10, 30, "none"), (10, 64, "none"), (10, 45, "gpruning")]


def nav_dir(name: str) -> Path:
    return HERE / f"nav_{name.split('_', 1)[1]}"


def make_navs() -> None:
    from quiver_b200 import builder
    for name, f in FIXTURES.items():
        base = builder.synth_mixture(f["seed"], f["n"], f["dim"], f["centers"], f["sigma"], f["dtype"])
        builder.build_nav(nav_dir(name), base, n_nav=NAV_SIZES[name], seed=f["seed"])


def make_reference_nav_outputs(out_dir: Path) -> None:
    from oracle import pyoracle, ref_harness
    from quiver_b200 import formats
    out_dir.mkdir(parents=True, exist_ok=True)
    for name, f in FIXTURES.items():
        ix = pyoracle.load_index(HERE / name, f["dtype"])
        nav = pyoracle.load_nav(nav_dir(name), f["dtype"])
        q = formats.read_bin(HERE / name / "queries.fbin", np.float32)
        arrays = {}
        for k, ef, pol in NAV_SETTINGS:
            r = ref_harness.run(ix, q, topk=k, ef_search=ef, early_exit_policy=pol, nav=nav)
            tag = f"k{k}_ef{ef}_{pol}"
            for key, val in r.items():
                arrays[f"{tag}_{key}"] = val
        np.savez(out_dir / f"ref_nav_{name}.npz", **arrays)
        print(f"wrote {out_dir / f'ref_nav_{name}.npz'}")


def make_indexes() -> None:
    from quiver_b200 import builder, formats
    for name, f in FIXTURES.items():
        d = HERE / name
        base = builder.synth_mixture(f["seed"], f["n"], f["dim"], f["centers"], f["sigma"], f["dtype"])
        q = builder.synth_mixture(f["seed"], f["nq"], f["dim"], f["centers"], f["sigma"], f["dtype"], stream=1)
        builder.build_index(d, base, R=f["R"], L=f["L"], alpha=1.2, M=f["M"], passes=2, pq_sample=f["n"],
                            seed=f["seed"], prefix="fixture")
        formats.write_bin(d / "queries.fbin", q.astype(np.float32))


def make_reference_outputs(out_dir: Path) -> None:
    from oracle import pyoracle, ref_harness
    out_dir.mkdir(parents=True, exist_ok=True)
    for name, f in FIXTURES.items():
        ix = pyoracle.load_index(HERE / name, f["dtype"])
        from quiver_b200 import formats
        q = formats.read_bin(HERE / name / "queries.fbin", np.float32)
        arrays = {}
        for k, ef, pol in SETTINGS:
            r = ref_harness.run(ix, q, topk=k, ef_search=ef, early_exit_policy=pol)
            tag = f"k{k}_ef{ef}_{pol}"
            for key, val in r.items():
                arrays[f"{tag}_{key}"] = val
        np.savez(out_dir / f"ref_{name}.npz", **arrays)
        print(f"wrote {out_dir / f'ref_{name}.npz'}")


if __name__ == "__main__":
    if sys.argv[1] == "index":
        make_indexes()
    elif sys.argv[1] == "nav":
        make_navs()
    elif sys.argv[1] == "refnav":
        make_reference_nav_outputs(Path(sys.argv[2]))
    else:
        make_reference_outputs(Path(sys.argv[2]))
