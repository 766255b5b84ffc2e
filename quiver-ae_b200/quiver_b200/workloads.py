"""The synthetic workloads of the benchmark configurations.

Each configuration is a seeded Gaussian mixture standing in for SIFT / DEEP
(which are not redistributable and not present here): same dimension,
element type, graph degree and PQ width as the named dataset shape.
Indexes are built once per cache directory and reused.
"""
from __future__ import annotations

import hashlib
import json
import os
import time
from dataclasses import asdict, dataclass
from pathlib import Path

import numpy as np

from . import builder, formats


@dataclass(frozen=True)
class Workload:
    name: str
    n: int
    dim: int
    data_type: str
    centers: int
    sigma: float
    R: int
    L: int
    alpha: float
    M: int
    nq: int
    topk: int
    ef_search: int
    seed: int = 0
    passes: int = 2
    pq_sample: int = 100_000


CONFIGS = {
    # 1M x 128-d uint8, 1000-cluster mixture (sigma 20), Vamana R=64 L=100 alpha=1.2,
    # PQ 32 x 256, 10K queries, top-10, ef_search=45, heap memory backend.
    "config0": Workload("config0", 1_000_000, 128, "uint8", 1000, 20.0, 64, 100, 1.2, 32, 10_000, 10, 45),
    # 10M x 96-d float32 unit-normalised, 5000 clusters (sigma 0.1), R=64, PQ 32 x 256.
    "config1": Workload("config1", 10_000_000, 96, "float", 5000, 0.1, 64, 100, 1.2, 32, 10_000, 10, 45),
    # 100M x 128-d uint8 mixture as config 0 with 10K clusters, R=64, PQ 32 x 256 (3.2 GB of
    # codes, 41 GB of graph pages -- both fit one B200's HBM), 100K queries per step, top-10.
    "config2": Workload("config2", 100_000_000, 128, "uint8", 10_000, 20.0, 64, 100, 1.2, 32, 100_000, 10, 45),
    # the first 10M rows of config 2's base stream (same 10K-cluster mixture, same query stream): config 2's
    # data at a size that builds in minutes, for recall diagnosis
    "config2-10m": Workload("config2-10m", 10_000_000, 128, "uint8", 10_000, 20.0, 64, 100, 1.2, 32, 10_000, 10, 45),
    # small shapes of config0 for tests and smoke runs
    "config0-100k": Workload("config0-100k", 100_000, 128, "uint8", 100, 20.0, 64, 100, 1.2, 32, 10_000, 10, 45),
    "config0-20k": Workload("config0-20k", 20_000, 128, "uint8", 20, 20.0, 64, 100, 1.2, 32, 2_000, 10, 45),
}


def cache_root() -> Path:
    return Path(os.environ.get("QUIVER_B200_CACHE", "/tmp/quiver_b200_cache"))


def index_dir(w: Workload) -> Path:
    return cache_root() / f"{w.name}-s{w.seed}"


def queries(w: Workload, rows: int | None = None, row0: int = 0, device: int | None = None) -> np.ndarray:
    n = w.nq if rows is None else rows
    return builder.synth_mixture(w.seed, n, w.dim, w.centers, w.sigma, w.data_type, stream=1, row0=row0,
                                 device=device)


def base(w: Workload, device: int | None = None) -> np.ndarray:
    """The base set; generated on GPU `device` when given (the same bits as on the host)."""
    return builder.synth_mixture(w.seed, w.n, w.dim, w.centers, w.sigma, w.data_type, stream=0, device=device)


def prepare(w: Workload, log=print, device: int | None = None) -> Path:
    """Build (or reuse) the index of `w`; returns its directory.  With a GPU `device` the data, the graph and
    the PQ codes are produced there (the same files as the host build)."""
    d = index_dir(w)
    stamp = d / "workload.json"
    if stamp.exists() and json.loads(stamp.read_text()) == asdict(w):
        return d
    d.mkdir(parents=True, exist_ok=True)
    t0 = time.time()
    b = base(w, device)
    where = "host" if device is None else f"GPU {device}"
    log(f"[workload] {w.name}: synthesised {w.n} x {w.dim} {w.data_type} on {where} in {time.time() - t0:.1f}s")
    t0 = time.time()
    builder.build_index(d, b, R=w.R, L=w.L, alpha=w.alpha, M=w.M, passes=w.passes, pq_sample=w.pq_sample,
                        seed=w.seed, device=device)
    build_s = time.time() - t0
    log(f"[workload] {w.name}: Vamana R={w.R} L={w.L} alpha={w.alpha} + PQ M={w.M} built on {where} in "
        f"{build_s:.1f}s")
    (d / "build.json").write_text(json.dumps({"where": where, "seconds": build_s}))
    stamp.write_text(json.dumps(asdict(w)))
    return d


def build_info(w: Workload) -> dict | None:
    """Where and how fast the cached index of `w` was built (None if unknown)."""
    p = index_dir(w) / "build.json"
    return json.loads(p.read_text()) if p.exists() else None


def prepare_nav(w: Workload, log=print) -> Path:
    """Build (or reuse) a nav graph for the index of `w` in its nav/ child
    (builder.build_nav defaults: a 1 % sample, degree 28)."""
    d = prepare(w, log=log)
    nav_dir = d / "nav"
    stamp = nav_dir / "nav.json"
    want = {"workload": asdict(w), "n_nav": 0, "seed": w.seed}
    if stamp.exists() and json.loads(stamp.read_text()) == want:
        return nav_dir
    t0 = time.time()
    nav = builder.build_nav(nav_dir, base(w), seed=w.seed)
    log(f"[workload] {w.name}: nav graph of {nav.graph.shape[0]} nodes built in {time.time() - t0:.1f}s")
    stamp.write_text(json.dumps(want))
    return nav_dir


def ground_truth(w: Workload, q: np.ndarray, k: int = 10, device: str | None = None) -> np.ndarray:
    """Exact top-k of `q` against the base set (GPU brute force when a device is given)."""
    d = index_dir(w)
    key = d / f"gt_{q.shape[0]}_{k}_{hashlib.sha1(q.tobytes()).hexdigest()[:12]}.ibin"
    if key.exists():
        return formats.read_bin(key, np.int32)
    if device is None:
        b = base(w)
        ids, _ = builder.ground_truth(b, q, k)
    else:
        b = base(w, int(str(device).split(":")[-1]))
        ids = _gt_torch(b, q, k, device)
    formats.write_bin(key, ids)
    return ids


def _gt_torch(b: np.ndarray, q: np.ndarray, k: int, device: str) -> np.ndarray:
    """Brute force on the GPU with an fp32 GEMM (TF32 off).  For uint8 data
    every product and partial sum of x.q is an integer below 2^24, so the
    distance ||x||^2 + ||q||^2 - 2 x.q is exact; float data is fp32.  Ties at
    the k-th place are broken by lower id within a base chunk."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out = np.empty((q.shape[0], k), dtype=np.int32)
        bchunk = 1 << 18
        qchunk = 2048
        xs = []
        for s in range(0, b.shape[0], bchunk):
            x = torch.from_numpy(b[s:s + bchunk].astype(np.float32)).to(device)
            xs.append((s, x, (x * x).sum(1)))
        for qs in range(0, q.shape[0], qchunk):
            qb = torch.from_numpy(q[qs:qs + qchunk].astype(np.float32)).to(device)
            qn = (qb * qb).sum(1, keepdim=True)
            best_d = torch.full((qb.shape[0], k), float("inf"), device=device)
            best_i = torch.zeros((qb.shape[0], k), dtype=torch.int64, device=device)
            for s, x, xn in xs:
                dot = torch.matmul(qb, x.T)
                assert dot.dtype == torch.float32
                dist = qn + xn[None, :] - 2 * dot
                td, ti = torch.topk(dist, min(k, dist.shape[1]), dim=1, largest=False, sorted=True)
                cand_d = torch.cat([best_d, td], 1)
                cand_i = torch.cat([best_i, ti + s], 1)
                order = torch.argsort(cand_i, dim=1)
                cand_d = torch.gather(cand_d, 1, order)
                cand_i = torch.gather(cand_i, 1, order)
                sd, si = torch.sort(cand_d, dim=1, stable=True)
                best_d = sd[:, :k]
                best_i = torch.gather(cand_i, 1, si[:, :k])
            out[qs:qs + qb.shape[0]] = best_i.to(torch.int32).cpu().numpy()
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
