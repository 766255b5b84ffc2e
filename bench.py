#!/usr/bin/env python
"""Throughput of Quiver's query hot path on B200.

One step = one search pass over one batch of synthetic queries (the
workload's step batch: 100K rows of its query stream for the default
config 2, 100M x 128 uint8; 10K for config 0) against the workload's index,
top-10, at the smallest ef_search from a fixed ladder whose Recall@10
reaches the target (0.90 by default).  The index is built on the GPU at the
start of the run and cached for later runs on the same machine.  Prints one
JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 runs under torchrun: each rank holds a replica of the index and
searches its own step batch (weak scaling, no collective on the data path;
the barrier and the max-over-ranks timing use NCCL).

Besides the headline (HBM page store), the line carries: ``latency_mode``
(batches of 1, 4 and 16 end to end), ``host_pages`` at N = 1 (node records
read over PCIe from pinned host DRAM, config 2's layout) and ``striped`` at
N > 1 (the page store striped over the ranks' GPUs and read over NVLink,
the 1B layout), each at the same ef and queries as the headline.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "quiver-ae_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "QPS at Recall@10=0.90 and P99 latency (ms), 1/2/4/8 B200, 1B×128 uint8"
# ef_search values tried in order, about 12 % apart above 100 so the smallest ef reaching the target is found
# closely; the engine accepts up to 4096
EF_LADDER = (45, 60, 80, 100, 112, 125, 140, 160, 180, 200, 225, 256, 288, 320, 360, 400, 450, 512, 576, 640, 720,
             800, 900, 1024, 1152, 1280, 1440, 1600, 1800, 2048, 2304, 2560, 2880, 3200, 3600, 4096)
CALIB_QUERIES = 2000
# where a configuration's own description puts the node records, when the headline uses another store
PAGE_STORE_NOTES = {
    "config2": "configs[2] lists the graph pages in pinned host DRAM; on a B200 its 41 GB fit in HBM, which the "
               "headline uses, and the host_pages object of the same line measures that layout (N = 1)",
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def entry_desc(nav_nodes: int) -> str:
    return f"nav graph entry search ({nav_nodes} nodes)" if nav_nodes else "medoid (no nav graph)"


def workload_desc(w) -> str:
    return (f"{w.name}: {w.n // 1_000_000 if w.n >= 1_000_000 else w.n}{'M' if w.n >= 1_000_000 else ''} x {w.dim}-d "
            f"{w.data_type} seeded {w.centers}-cluster Gaussian mixture (sigma {w.sigma}); Vamana R={w.R} "
            f"L={w.L} alpha={w.alpha}; PQ M={w.M} x 256; {w.nq} queries per step; top-{w.topk}")


def pick_ef(recall_of, target: float) -> tuple[int, float]:
    """Smallest ladder ef whose Recall@10 reaches the target (else the largest)."""
    r = 0.0
    for ef in EF_LADDER:
        r = recall_of(ef)
        if r >= target:
            return ef, r
    return EF_LADDER[-1], r


def read_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def read_nvlink_peak() -> dict:
    """Per-direction NVLink peer bandwidth per GPU: MEASURED_PEAKS.json's figure when it has one, else the
    pool's measured peer copy (770 GB/s per direction; 900 nominal)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        for key in ("nvlink_gbs", "p2p_gbs"):
            if key in d:
                return {"gbs": float(d[key]), "source": "measured"}
    return {"gbs": 770.0, "source": "pool peer-copy measurement (fallback)"}


def time_steps(eng, dq, p, d_ids, d_dists, stream, steps: int, warmup: int, barrier, device):
    """`warmup` untimed launches, then `steps` timed ones with CUDA events on `stream`, bracketed by barriers;
    returns (per-step ms on this rank, max over ranks of the total ms)."""
    import torch
    from quiver_b200 import shard
    for _ in range(warmup):
        eng.search_device(dq, p, d_ids, d_dists, stream=stream.cuda_stream)
    barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    evs[0].record(stream)
    for i in range(steps):
        eng.search_device(dq, p, d_ids, d_dists, stream=stream.cuda_stream)
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    eng.check_device_status()
    step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
    total_ms = shard.reduce_max(evs[0].elapsed_time(evs[-1]), device=device)
    barrier()
    return step_ms, total_ms


def pcie_h2d_gbs(dev) -> float:
    """Host-to-device copy rate of a pinned 1 GiB buffer on this box (best of 3, CUDA events)."""
    import torch
    src = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    best = float("inf")
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dst.copy_(src, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del src, dst
    return (1 << 30) / (best / 1000.0) / 1e9


def read_profile_traffic(name: str) -> float | None:
    """dram bytes per launch from a committed ncu summary (key: value lines)."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch_scaled:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.tmp = None

    def __enter__(self):
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.device), "-lms", "100"], stdout=self.tmp,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in Path(self.tmp.name).read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        finally:
            os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def reference_arm(args, rank: int, world: int) -> int:
    """The reference's CPU implementation of the path, on the host cores.

    The reference ships no CPU search (its DiskANN submodule is empty), so
    this arm runs the oracle -- the C restatement of the reference kernel's
    semantics -- with every host thread, on the same index, queries and ef."""
    if rank != 0:
        return 0
    from oracle import pyoracle
    from quiver_b200 import workloads
    w = workloads.CONFIGS[args.config]
    # the index is the search's input: build it on the GPU when there is one (the same files as a host build)
    try:
        import torch
        build_dev = 0 if torch.cuda.is_available() else None
    except ImportError:
        build_dev = None
    d = workloads.prepare(w, log=log, device=build_dev)
    ix = pyoracle.load_index(d, w.data_type)
    nav = pyoracle.load_nav(workloads.prepare_nav(w, log=log), w.data_type) if args.nav else None
    qc = workloads.queries(w, rows=CALIB_QUERIES).astype(np.float32)
    # ground truth, like the index, is an input: brute force on the GPU when there is one
    gtc = workloads.ground_truth(w, qc, 10, device=None if build_dev is None else f"cuda:{build_dev}")
    search_kw = dict(topk=w.topk, pipe_width=args.pipe_width, early_exit_policy=args.early_exit, nav=nav,
                     visited_filter=args.visited_filter)
    if args.ef > 0:
        ef = args.ef
        recall = pyoracle.calc_recall(pyoracle.search(ix, qc, ef_search=ef, **search_kw)["ids"], gtc, 10)
    else:
        ef, recall = pick_ef(lambda e: pyoracle.calc_recall(pyoracle.search(ix, qc, ef_search=e, **search_kw)["ids"],
                                                            gtc, 10), args.target_recall)
    q = workloads.queries(w).astype(np.float32)
    cores = os.cpu_count() or 1
    # size each step to ~0.5 s of host work so K steps end within minutes
    t = time.perf_counter()
    pyoracle.search(ix, q[:256], ef_search=ef, **search_kw)
    rate = 256 / max(time.perf_counter() - t, 1e-6)
    per_step = int(min(w.nq, max(64, rate * 0.5)))
    for i in range(args.warmup):
        pyoracle.search(ix, q[:per_step], ef_search=ef, **search_kw)
    t = time.perf_counter()
    for i in range(args.steps):
        s0 = (i * per_step) % max(1, w.nq - per_step + 1)
        pyoracle.search(ix, q[s0:s0 + per_step], ef_search=ef, **search_kw)
    dt = time.perf_counter() - t
    qps = args.steps * per_step / dt
    sample = f"{per_step} of the {w.nq} queries per step, ef_search={ef}, pipe_width={args.pipe_width}"
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1000 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture; SIFT/DEEP not present)",
        "config": {"workload": workload_desc(w), "ef_search": ef, "recall_at_10": recall,
                   "pipe_width": args.pipe_width, "early_exit": args.early_exit,
                   "entry": entry_desc(nav.graph.shape[0] if nav is not None else 0),
                   "visited_filter": args.visited_filter},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "recall_at_10": recall,
        "note": ("timed: the oracle's search only (the C restatement of the reference kernel, all host threads), "
                 "on a bounded sample of each step's queries; the index it searches -- its input -- is built "
                 "beforehand by this repository's GPU builder, bit-identical to the host build"),
    }
    print(json.dumps(line), flush=True)
    return 0


CPU_SAMPLE_SECONDS, CPU_SAMPLE_MAX_ROWS = 12.0, 200_000


def cpu_baseline(w, d, ef: int, args, seconds: float = CPU_SAMPLE_SECONDS) -> dict:
    """The oracle on a bounded sample, all host threads, N=1 rank 0 only.  The sample is sized for about
    `seconds` of host work from a 256-query calibration: the first rows of the seeded query stream (the step
    batch first, then further rows of the same mixture when one batch is too little work)."""
    from oracle import pyoracle
    from quiver_b200 import workloads
    ix = pyoracle.load_index(d, w.data_type)
    nav = pyoracle.load_nav(d / "nav", w.data_type) if args.nav else None
    kw = dict(topk=w.topk, ef_search=ef, pipe_width=args.pipe_width, early_exit_policy=args.early_exit, nav=nav,
              visited_filter=args.visited_filter)
    q = workloads.queries(w, rows=256).astype(np.float32)
    t = time.perf_counter()
    pyoracle.search(ix, q, **kw)
    rate = 256 / max(time.perf_counter() - t, 1e-6)
    n = int(min(CPU_SAMPLE_MAX_ROWS, max(256, rate * seconds)))
    q = workloads.queries(w, rows=n).astype(np.float32)
    t = time.perf_counter()
    pyoracle.search(ix, q, **kw)
    dt = time.perf_counter() - t
    rows = (f"the first {n} of the {w.nq} step queries" if n <= w.nq else
            f"the {w.nq} step queries and the next {n - w.nq} rows of the same seeded query stream")
    return {"value": n / dt, "unit": "queries/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{rows}, ef_search={ef}, {dt:.1f} s of host work"}


def host_pages_pass(args, w, d, local, dev, dq, p, d_ids, d_dists, stream, barrier, nq, rec_bytes, recall) -> dict:
    """The headline step again with the page store in pinned host DRAM mapped into the GPU (QV_PAGES_HOST):
    node records cross PCIe, everything else stays in HBM.  Same resident queries, ef and pipe width."""
    import torch
    from quiver_b200 import Engine
    ref_ids = d_ids.clone()
    with Engine.open(d, w.data_type, device=local, page_store="host") as eh:
        h_ms, h_total = time_steps(eh, dq, p, d_ids, d_dists, stream, args.steps, args.warmup, barrier, dev)
        same = bool(torch.equal(d_ids, ref_ids))
    pcie_peak = pcie_h2d_gbs(dev)
    gbs = rec_bytes / (statistics.mean(h_ms) / 1000.0) / 1e9
    return {"qps": args.steps * nq / (h_total / 1000.0), "ms_per_step": h_total / args.steps,
            "ids_equal_to_hbm_store": same, "recall_at_10": recall if same else None,
            "record_bytes_per_step": rec_bytes, "pcie_gbs": gbs, "pcie_peak_gbs": pcie_peak,
            "pcie_frac": gbs / pcie_peak,
            "how": "qv_search_device on the same resident queries with QV_PAGES_HOST (the page store in pinned "
                   "host DRAM mapped into the GPU, records read by the kernel over PCIe); record bytes = "
                   "expansions x node_size; peak = a pinned 1 GiB host-to-device copy timed in this run"}


def striped_pass(args, w, d, local, dev, dq, p, d_ids, d_dists, stream, barrier, nq, world, rec_bytes,
                 replicated_qps) -> dict:
    """The headline step with the page store striped over the ranks (QV_PAGES_SHARED: page p on rank p mod N,
    opened by CUDA IPC, read with plain peer loads).  Every rank takes the same collective steps, failures
    included: each local step (open this rank's stripe, attach the others) is followed by an all-reduce of
    its success, so a rank that fails makes every rank skip the rest instead of leaving the others blocked,
    and the headline line is kept with an `error` here."""
    import torch
    import torch.distributed as dist
    from quiver_b200 import Engine, shard

    def all_ok(ok: bool) -> bool:
        t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return bool(t.item())

    ref_ids = d_ids.clone()
    es, err = None, None
    try:
        es = Engine.open(d, w.data_type, device=local, page_store="shared", num_stripes=world,
                         stripe_rank=dist.get_rank())
    except Exception as e:  # noqa: BLE001 -- reported in the line
        err = f"open: {type(e).__name__}: {e}"
    if not all_ok(es is not None):
        if es is not None:
            es.close()
        return {"error": err or "another rank could not open its stripe"}
    handles = shard.exchange_stripe_handles(es.stripe_handle())
    try:
        es.attach_stripes(handles)
        attached = True
    except Exception as e:  # noqa: BLE001
        err, attached = f"attach: {type(e).__name__}: {e}", False
    if not all_ok(attached):
        barrier()
        es.close()
        return {"error": err or "another rank could not attach the stripes"}
    s_ms, s_total = time_steps(es, dq, p, d_ids, d_dists, stream, args.steps, args.warmup, barrier, dev)
    same = all_ok(bool(torch.equal(d_ids, ref_ids)))
    remote = torch.tensor([rec_bytes * (world - 1) / world / (statistics.mean(s_ms) / 1000.0)], dtype=torch.float64,
                          device=dev)
    dist.all_reduce(remote, op=dist.ReduceOp.SUM)
    barrier()  # every rank reads every other rank's stripe: close only when all are done
    es.close()
    s_value = world * args.steps * nq / (s_total / 1000.0)
    nvl = read_nvlink_peak()
    per_gpu = float(remote.item()) / world / 1e9
    return {"qps": s_value, "ms_per_step": s_total / args.steps, "efficiency_vs_replicated": s_value / replicated_qps,
            "ids_equal_to_replicated": same, "nvlink_gbs_per_gpu": per_gpu,
            "nvlink_peak_gbs": nvl["gbs"], "nvlink_peak_source": nvl["source"], "nvlink_frac": per_gpu / nvl["gbs"],
            "how": "QV_PAGES_SHARED: page p on rank p mod N (CUDA IPC, plain peer loads); remote record bytes = "
                   "expansions x node_size x (N-1)/N per rank over its mean step time, averaged over ranks"}


ADC_POINTS, ADC_QUERIES, ADC_PER_QUERY = 100_000_000, 2048, 65_536
# (mode, kernel, algorithmic bytes per pair): 32 code + 4 distance written, + 4 id read for gathers
ADC_DEFAULT = (("stream", "pipe", 36), ("gather", "thread", 40))
ADC_ALL = (("stream", "pipe", 36), ("stream", "thread", 36), ("gather", "thread", 40), ("gather", "pipe", 40))


def adc_microbench(dev, stream, peak_gbs: float, points: int = ADC_POINTS, queries: int = ADC_QUERIES,
                   per_query: int = ADC_PER_QUERY, reps: int = 10, combos=ADC_DEFAULT) -> dict:
    """Batched ADC (qv_adc_batch) over `points` x 32-byte codes in HBM (100M = 3.2 GB, config 2's code
    array, by default): `queries` x `per_query` codes, as contiguous ranges (stream) and as uniformly random
    ids (gather).  Every combination is warmed up (3 launches each, in order) before any is timed, then each
    is timed over `reps` launches with CUDA events on `stream`."""
    import torch
    from quiver_b200.adc import adc_batch
    g = torch.Generator(device=dev).manual_seed(7)
    codes = torch.empty((points, 32), dtype=torch.uint8, device=dev)
    step = 10_000_000
    for i in range(0, points, step):
        codes[i:i + step] = torch.randint(0, 256, (min(step, points - i), 32), dtype=torch.uint8, device=dev,
                                          generator=g)
    luts = torch.rand((queries, 32, 256), device=dev, generator=g) * 4096.0
    first = (torch.arange(queries, device=dev, dtype=torch.int64) * per_query) % (points - per_query)
    ids = torch.randint(0, points, (queries, per_query), dtype=torch.int32, device=dev, generator=g)
    out = torch.empty((queries, per_query), dtype=torch.float32, device=dev)
    pairs = queries * per_query
    res = {"workload": f"{points / 1e6:g}M codes x 32 B in HBM ({points * 32 / 1e9:.2f} GB), {queries} queries x "
                       f"{per_query} codes, fp32 LUTs, chunk-ordered sums",
           "peak_gbs": peak_gbs}

    def run(mode, kernel):
        if mode == "stream":
            adc_batch(codes, luts, first=first, n_per_query=per_query, out=out, kernel=kernel, stream=stream)
        else:
            adc_batch(codes, luts, ids, out=out, kernel=kernel, stream=stream)

    for mode, kernel, _ in combos:
        for _ in range(3):
            run(mode, kernel)
    for mode, kernel, per_pair in combos:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            run(mode, kernel)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        gbs = pairs * per_pair / (ms / 1e3) / 1e9
        key = mode if combos is ADC_DEFAULT else f"{mode}_{kernel}"
        res[key] = {"kernel": f"adc_{kernel}", "ms_per_launch": ms, "gpairs_per_s": pairs / (ms / 1e3) / 1e9,
                    "alg_bytes_per_pair": per_pair, "achieved_gbs": gbs, "frac": gbs / peak_gbs,
                    "code_gbs": pairs * 32 / (ms / 1e3) / 1e9}
    del codes, luts, first, ids, out
    torch.cuda.empty_cache()
    return res


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="config2",
                    help="workload (quiver_b200.workloads.CONFIGS); config2, the metric's largest single-GPU "
                         "configuration, builds its index on the GPU first (about 5 minutes)")
    ap.add_argument("--ef", type=int, default=0, help="fixed ef_search (0: smallest ladder ef reaching the target)")
    ap.add_argument("--target-recall", type=float, default=0.90)
    ap.add_argument("--pipe-width", type=int, default=2)
    ap.add_argument("--early-exit", default="none", choices=["none", "gpruning"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--latency", default="1,4,16",
                    help="also time small batches end to end (latency mode, the batches of config 4; rank 0 "
                         "only); empty to skip")
    ap.add_argument("--no-host-pages", action="store_true",
                    help="skip the host-DRAM page store pass (host_pages object, N = 1)")
    ap.add_argument("--no-striped", action="store_true",
                    help="skip the shared striped page store pass (striped object, N > 1)")
    ap.add_argument("--stripe-devices", default="",
                    help="stripe the page store over these GPUs, e.g. 0,1 (pages p mod S; peer loads)")
    ap.add_argument("--page-store", default="hbm", choices=["hbm", "host"],
                    help="where the node records live: the search GPU's HBM, or pinned host DRAM mapped into the "
                         "GPU's address space and read over PCIe")
    ap.add_argument("--stripe-shared", action="store_true",
                    help="under torchrun: rank r holds pages p = r (mod N) and reads the rest from the other "
                         "ranks' GPUs (CUDA IPC, peer loads)")
    ap.add_argument("--visited-filter", action="store_true",
                    help="the engine's visited-filter mode (not reference behaviour; reports its recall)")
    ap.add_argument("--nav", action="store_true",
                    help="start each query from the nav-graph entry search (a 1 %% nav graph is built and cached)")
    ap.add_argument("--no-stream", action="store_true",
                    help="skip the streaming-admission measurement (profilers that serialise kernels and copies, "
                         "such as ncu, stall its feed)")
    ap.add_argument("--no-adc", action="store_true",
                    help="skip the batched-ADC measurement (adc_batch object of the JSON line)")
    ap.add_argument("--adc-only", action="store_true",
                    help="run only the batched-ADC measurement, every kernel on both access patterns")
    ap.add_argument("--adc-points", type=int, default=ADC_POINTS)
    ap.add_argument("--adc-queries", type=int, default=ADC_QUERIES)
    ap.add_argument("--adc-reps", type=int, default=10)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # torchrun pins every rank to one OpenMP thread; the host-side work here
    # (the index build on rank 0 while the other ranks wait, the reference
    # arm on rank 0 alone) should use every core.  Set before any native
    # library with OpenMP is loaded.
    if "LOCAL_RANK" in os.environ and os.environ.get("OMP_NUM_THREADS") == "1":
        os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist
    from quiver_b200 import Engine, SearchParams, shard, workloads

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.adc_only:
        if rank == 0:
            stream = torch.cuda.Stream(dev)
            res = adc_microbench(dev, stream, read_peaks()["hbm_gbs"], points=args.adc_points,
                                 queries=args.adc_queries, reps=args.adc_reps, combos=ADC_ALL)
            print(json.dumps({"adc_batch": res}), flush=True)
        return 0
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    w = workloads.CONFIGS[args.config]
    if rank == 0:
        workloads.prepare(w, log=log, device=local)
        if args.nav:
            workloads.prepare_nav(w, log=log)
    barrier()
    d = workloads.index_dir(w)
    stripes = [int(x) for x in args.stripe_devices.split(",") if x]
    if args.stripe_shared:
        eng = shard.open_shared(d, w.data_type, device=local)
    elif stripes:
        eng = Engine.open(d, w.data_type, device=local, page_store="striped", stripe_devices=stripes)
    else:
        eng = Engine.open(d, w.data_type, device=local, page_store=args.page_store)
    nav_nodes = eng.nav_info[0] if args.nav else 0

    # ef calibration on the first CALIB_QUERIES rows (identical on every rank)
    qc = workloads.queries(w, rows=CALIB_QUERIES)
    if rank == 0:
        workloads.ground_truth(w, qc, 10, device=f"cuda:{local}")
    barrier()
    gtc = workloads.ground_truth(w, qc, 10)
    from quiver_b200.recall import calc_recall

    def params(ef):
        return SearchParams(topk=w.topk, ef_search=ef, pipe_width=args.pipe_width, early_exit_policy=args.early_exit,
                            skip_nav=not args.nav, visited_filter=args.visited_filter)

    def recall_of(ef):
        return calc_recall(eng.search(qc, params(ef))[0], gtc, 10)

    if args.ef > 0:
        ef, recall = args.ef, recall_of(args.ef)
    else:
        ef, recall = pick_ef(recall_of, args.target_recall)
    p = params(ef)

    # this rank's step batch, resident in HBM
    row0, rows = shard.weak_rows(rank, w.nq)
    q = workloads.queries(w, rows=rows, row0=row0).astype(np.float32)
    nq, k = q.shape[0], w.topk
    dq = torch.from_numpy(q).to(dev)
    d_ids = torch.empty((nq, k), dtype=torch.int32, device=dev)
    d_dists = torch.empty((nq, k), dtype=torch.float32, device=dev)
    d_steps = torch.empty(nq, dtype=torch.int32, device=dev)
    d_nbrs = torch.empty(nq, dtype=torch.int64, device=dev)
    stream = torch.cuda.Stream(dev)  # every launch, event and copy of the step runs here
    torch.cuda.set_stream(stream)

    # algorithmic bytes of one launch: query rows, node records, PQ codes gathered, results
    eng.search_device(dq, p, d_ids, d_dists, None, d_steps, d_nbrs, stream=stream.cuda_stream)
    torch.cuda.synchronize()
    eng.check_device_status()
    info = eng.info
    expansions = int(d_steps.sum().item())
    gathered = int(d_nbrs.sum().item())
    alg_bytes = nq * (4 * info.dim + 8 * k) + expansions * info.node_size + gathered * info.num_chunks

    for _ in range(args.warmup):
        eng.search_device(dq, p, d_ids, d_dists, stream=stream.cuda_stream)
    barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(local) as clk:
        evs[0].record(stream)
        for i in range(args.steps):
            eng.search_device(dq, p, d_ids, d_dists, stream=stream.cuda_stream)
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
    clocks = clk.summary()
    eng.check_device_status()
    step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    total_ms = shard.reduce_max(evs[0].elapsed_time(evs[-1]), device=dev)
    barrier()
    value = world * args.steps * nq / (total_ms / 1000.0)

    # per-query service latency at the same operating point (kernel timer: bind to finish)
    lat = eng.search_timed(q, p)[3]
    p50, p99 = float(np.percentile(lat, 50)), float(np.percentile(lat, 99))

    # streaming admission: the reference's host loop and its QueryLatency(ms)
    # (admission to observed completion); the call with the median QPS of 5
    streaming = None
    if rank == 0 and not args.no_stream:
        eng.search_stream(q, p)
        runs = sorted((eng.search_stream(q, p)[4] for _ in range(5)), key=lambda st: st.qps)
        st = runs[len(runs) // 2]
        streaming = {"qps": st.qps, "lat_avg_ms": st.lat_avg_ms, "p50_ms": st.lat_p50_ms, "p90_ms": st.lat_p90_ms,
                     "p99_ms": st.lat_p99_ms, "p999_ms": st.lat_p999_ms, "max_ms": st.lat_max_ms,
                     "workers": st.workers, "max_inflight": st.max_inflight, "admissions": st.admissions,
                     "queries": nq,
                     "how": "qv_search_stream: one persistent launch, host admits ranges as completions allow "
                            "(prefeed = workers, admit_min_batch 32); latency = host time from a query's "
                            "admission to the completion count passing it; median-QPS call of 5"}

    # end to end through the C ABI with pinned host buffers
    hq = torch.from_numpy(q).pin_memory()
    h_ids = torch.empty((nq, k), dtype=torch.int32).pin_memory()
    h_dists = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    for _ in range(2):
        eng.search_host_ptrs(hq.data_ptr(), nq, info.dim, p, h_ids.data_ptr(), h_dists.data_ptr())
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.search_host_ptrs(hq.data_ptr(), nq, info.dim, p, h_ids.data_ptr(), h_dists.data_ptr())
    e2e_s = shard.reduce_max(time.perf_counter() - t0, device=dev)
    barrier()
    step_recall = calc_recall(h_ids.numpy(), workloads.ground_truth(w, q, 10, device=f"cuda:{local}"), 10) \
        if rank == 0 else None

    # latency mode: batches of a few queries through qv_search (pinned host
    # buffers in and out, one kernel per batch), wall time per batch
    latency = {}
    if args.latency and rank == 0:
        for b in (int(x) for x in args.latency.split(",") if x):
            reps = max(50, 1000 // b)
            times = []
            for r in range(reps + 5):
                r0 = (r * b) % (nq - b + 1)
                t1 = time.perf_counter()
                eng.search_host_ptrs(hq[r0:].data_ptr(), b, info.dim, p, h_ids.data_ptr(), h_dists.data_ptr())
                if r >= 5:
                    times.append((time.perf_counter() - t1) * 1e3)
            latency[str(b)] = {"batches": reps, "p50_ms": float(np.percentile(times, 50)),
                               "p99_ms": float(np.percentile(times, 99)), "qps": b * 1e3 / statistics.mean(times)}

    # host-DRAM page store (config 2's layout): the same step with node records read over PCIe from pinned,
    # mapped host memory; everything else in HBM.  N = 1 only.
    host_pages = None
    if world == 1 and not args.no_host_pages and args.page_store == "hbm" and not stripes and not args.stripe_shared:
        try:
            host_pages = host_pages_pass(args, w, d, local, dev, dq, p, d_ids, d_dists, stream, barrier, nq,
                                         expansions * info.node_size, recall)
        except Exception as err:  # the headline stands without it (e.g. not enough pinnable host memory)
            host_pages = {"error": f"{type(err).__name__}: {err}"}

    # shared striped page store (the 1B layout): rank r holds pages p = r (mod N) in its HBM and reads the
    # other ranks' pages over NVLink with peer loads; the same per-rank step batch.  N > 1, every rank.
    striped = None
    if world > 1 and not args.no_striped and not args.stripe_shared and not stripes:
        striped = striped_pass(args, w, d, local, dev, dq, p, d_ids, d_dists, stream, barrier, nq, world,
                               expansions * info.node_size, value)

    if rank == 0:
        peaks = read_peaks()
        avg_ms = statistics.mean(step_ms)
        achieved = alg_bytes / (avg_ms / 1000.0) / 1e9
        traffic = read_profile_traffic(f"search_kernel_{w.name}.txt")
        line = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Gaussian mixture; SIFT/DEEP not present)",
            "config": {"workload": workload_desc(w), "ef_search": ef, "recall_at_10": recall,
                       "entry": entry_desc(nav_nodes), "visited_filter": args.visited_filter,
                       "recall_at_10_step_batch": step_recall, "pipe_width": args.pipe_width,
                       "early_exit": args.early_exit, "queries_per_step_per_gpu": nq,
                       "l2": f"inputs larger than L2: page store {info.num_pages * 4096 / 1e6:.0f} MB + codes "
                             f"{info.num_points * info.num_chunks / 1e6:.0f} MB vs 126 MB L2, no flush",
                       "parallelism": f"query shards x{world}, index replicated",
                       "index_build": workloads.build_info(w),
                       "page_store": (f"shared: rank r holds pages p = r mod {world}, the rest read from the other "
                                      f"ranks' GPUs (CUDA IPC peer loads)" if args.stripe_shared
                                      else f"striped over GPUs {stripes} (peer loads)" if stripes
                                      else "pinned host DRAM, mapped (PCIe loads)" if args.page_store == "host"
                                      else "HBM of the search GPU"),
                       "page_store_note": PAGE_STORE_NOTES.get(w.name)},
            "recall_at_10": recall,
            "p50_ms": streaming["p50_ms"] if streaming else p50,
            "p99_ms": streaming["p99_ms"] if streaming else p99,
            "latency_definition": ("QueryLatency(ms) of the streaming admission loop (see streaming)" if streaming
                                   else "kernel-timer service latency (streaming skipped)"),
            "streaming": streaming,
            "service_latency": {"p50_ms": p50, "p99_ms": p99,
                                "how": "kernel global timer from a worker binding the query to its results, "
                                       "every query admitted at the call (qv_search_timed)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"],
                         "traffic": traffic, "algorithmic_bytes_per_launch": alg_bytes,
                         "expansions_per_query": expansions / nq, "codes_per_query": gathered / nq},
            "e2e": {"value": world * args.steps * nq / e2e_s, "unit": "queries/s",
                    "h2d_bytes_per_step": int(q.nbytes), "d2h_bytes_per_step": int(nq * k * 8)},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
        if args.page_store == "host" and not stripes and not args.stripe_shared:
            # the committed capture is of the HBM page store; here the records come over PCIe
            line["roofline"]["traffic"] = None
            line["roofline"]["note"] = (f"node records ({expansions * info.node_size / 1e9:.2f} GB per launch) are read "
                                        "from pinned host DRAM over PCIe; the HBM fraction does not bound this mode")
        if host_pages:
            line["host_pages"] = host_pages
        if striped:
            line["striped"] = striped
        if latency:
            line["latency_mode"] = {"per_batch_size": latency,
                                    "how": "qv_search on pinned host buffers, host wall time per batch "
                                           "(H2D, one kernel, D2H, sync), same ef / pipe width"}
        if world == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline(w, d, ef, args)
            except Exception as err:  # e.g. the host cannot hold a second copy of a large index
                line["cpu_baseline"] = {"error": f"{type(err).__name__}: {err}"}
        if not args.no_adc:
            line["adc_batch"] = adc_microbench(dev, stream, peaks["hbm_gbs"])
        print(json.dumps(line), flush=True)
    if args.stripe_shared:
        barrier()  # every rank reads every other rank's stripe: close only when all are done
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
