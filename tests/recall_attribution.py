#!/usr/bin/env python
"""Where does Recall@10 go?  PQ routing against exact routing on one graph.

Diagnostic, not a test (pytest does not collect it).  For a benchmark
workload it builds (or reuses) the index on a GPU, then walks the SAME graph
with the oracle twice per ef_search: once as the reference does (neighbours
scored by PQ asymmetric distance, the exact L2 only for expanded nodes) and
once with every neighbour scored by its exact L2 (the oracle's route_exact
diagnostic).  The gap between the two recalls is what PQ costs; what the
exact walk still misses is the graph's (and the beam's) share.  Optionally it
also reports the CUDA engine's recall on the same queries (equal to the
oracle's PQ walk by the parity tests) for a longer ef ladder.

  python tests/recall_attribution.py --config config0 --queries 1000 --efs 45,100,200,320
  python tests/recall_attribution.py --config config2-10m --engine-efs 320,640,1024,2048,4096

Prints one JSON object per line.
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT / "quiver-ae_b200"), str(ROOT)]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="config0")
    ap.add_argument("--queries", type=int, default=1000)
    ap.add_argument("--efs", default="45,100,200,320")
    ap.add_argument("--engine-efs", default="", help="also the engine's recall at these ef (GPU)")
    ap.add_argument("--pipe-width", type=int, default=2)
    ap.add_argument("--device", type=int, default=0, help="GPU for the build and ground truth; -1: host only")
    args = ap.parse_args()

    from oracle import pyoracle
    from quiver_b200 import workloads
    from quiver_b200.recall import calc_recall
    w = workloads.CONFIGS[args.config]
    t0 = time.time()
    dev = None if args.device < 0 else args.device
    d = workloads.prepare(w, log=lambda *a: print(*a, file=sys.stderr, flush=True), device=dev)
    print(json.dumps({"config": w.name, "n": w.n, "build": workloads.build_info(w),
                      "prepare_s": time.time() - t0}), flush=True)
    q = workloads.queries(w, rows=args.queries).astype(np.float32)
    gt = workloads.ground_truth(w, q, 10, device=None if dev is None else f"cuda:{dev}")
    ix = pyoracle.load_index(d, w.data_type)
    for ef in (int(x) for x in args.efs.split(",") if x):
        row = {"config": w.name, "ef_search": ef, "pipe_width": args.pipe_width, "queries": len(q)}
        for mode, exact in (("pq_routing", False), ("exact_routing", True)):
            t = time.perf_counter()
            out = pyoracle.search(ix, q, topk=10, ef_search=ef, pipe_width=args.pipe_width,
                                  early_exit_policy="none", route_exact=exact)
            row[mode] = {"recall_at_10": calc_recall(out["ids"], gt, 10),
                         "expansions_per_query": float(out["steps"].mean()), "host_s": time.perf_counter() - t}
        print(json.dumps(row), flush=True)
    if args.engine_efs:
        from quiver_b200 import Engine, SearchParams
        with Engine.open(d, w.data_type, device=args.device) as eng:
            for ef in (int(x) for x in args.engine_efs.split(",") if x):
                p = SearchParams(topk=10, ef_search=ef, pipe_width=args.pipe_width, early_exit_policy="none")
                ids, _, _, st = eng.search(q, p, with_stats=True)
                print(json.dumps({"config": w.name, "engine_ef_search": ef, "queries": len(q),
                                  "recall_at_10": calc_recall(ids, gt, 10),
                                  "expansions_per_query": st.expansions / len(q)}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
