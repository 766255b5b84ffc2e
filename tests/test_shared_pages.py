"""Page store shared by the processes of a job (QV_PAGES_SHARED).

Rank r of S holds pages p = r (mod S) in its own GPU's HBM and reads the
other stripes from the processes that hold them (CUDA IPC).  The handle
exchange is host logic and runs here on gloo ranks; on a GPU, S processes
(on one GPU, or one per GPU when there are enough) must reproduce the
single-engine results bit for bit.  No kernel waits on another process.
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "quiver-ae_b200"), str(root)]
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    return dist


def _exchange_worker(rank: int, world: int, port: int, out: dict):
    dist = _init(rank, world, port)
    from quiver_b200 import shard
    got = shard.exchange_stripe_handles(bytes([rank]) * 64)
    out[rank] = got
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_stripe_handles_reach_every_rank_in_order(world):
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:  # no fork of a process that may hold a CUDA context
        out = m.dict()
        mp.spawn(_exchange_worker, args=(world, port, out), nprocs=world, join=True)
        for r in range(world):
            assert out[r] == [bytes([s]) * 64 for s in range(world)]


def _search_worker(rank: int, world: int, port: int, index_dir: str, queries: np.ndarray, per_gpu: bool,
                   out: dict):
    dist = _init(rank, world, port)
    import torch
    from quiver_b200 import Engine, QuiverEngineError, SearchParams, shard
    device = rank if per_gpu else 0
    torch.cuda.set_device(device)
    eng = Engine.open(index_dir, "uint8", device=device, page_store="shared", num_stripes=world, stripe_rank=rank)
    p = SearchParams(topk=10, ef_search=48, pipe_width=2, early_exit_policy="none")
    try:
        eng.search(queries[:4], p)
        out[f"early{rank}"] = "searched"
    except QuiverEngineError as e:
        out[f"early{rank}"] = str(e)
    eng.attach_stripes(shard.exchange_stripe_handles(eng.stripe_handle()))
    ids, dists, _ = eng.search(queries, p)
    q2 = torch.tensor(queries[:3], device=f"cuda:{device}")
    ids_t = torch.arange(0, 3000, 31, dtype=torch.int32, device=f"cuda:{device}")
    qof = (torch.arange(ids_t.numel(), device=f"cuda:{device}") % 3).to(torch.int32)
    l2 = torch.empty(ids_t.numel(), dtype=torch.float32, device=f"cuda:{device}")
    eng.exact_l2(q2, qof, ids_t, l2)
    torch.cuda.synchronize()
    out[rank] = (ids, dists, l2.cpu().numpy())
    dist.barrier()  # nobody closes its stripe while another rank may still read it
    eng.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world,per_gpu", [(2, False), (4, False), (2, True)])
def test_shared_store_equals_plain(u8_index, world, per_gpu):
    import torch
    from quiver_b200 import Engine, SearchParams
    if per_gpu and torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    q = u8_index["queries"]
    p = SearchParams(topk=10, ef_search=48, pipe_width=2, early_exit_policy="none")
    with Engine.open(u8_index["dir"], "uint8") as eng:
        ids, dists, _ = eng.search(q, p)
        q2 = torch.tensor(q[:3], device="cuda")
        ids_t = torch.arange(0, 3000, 31, dtype=torch.int32, device="cuda")
        qof = (torch.arange(ids_t.numel(), device="cuda") % 3).to(torch.int32)
        l2 = torch.empty(ids_t.numel(), dtype=torch.float32, device="cuda")
        eng.exact_l2(q2, qof, ids_t, l2)
        torch.cuda.synchronize()
        l2 = l2.cpu().numpy()
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        mp.start_processes(_search_worker, args=(world, port, str(u8_index["dir"]), q, per_gpu, out), nprocs=world,
                           join=True, start_method="spawn")
        for r in range(world):
            assert "qv_engine_attach_stripes" in out[f"early{r}"]
            got_ids, got_d, got_l2 = out[r]
            np.testing.assert_array_equal(got_ids, ids)
            np.testing.assert_array_equal(got_d.view(np.uint32), dists.view(np.uint32))
            np.testing.assert_array_equal(got_l2.view(np.uint32), l2.view(np.uint32))


@pytest.mark.gpu
def test_shared_store_argument_errors(u8_index):
    from quiver_b200 import Engine, QuiverEngineError
    with pytest.raises(QuiverEngineError, match="stripe_rank"):
        Engine.open(u8_index["dir"], "uint8", page_store="shared", num_stripes=2, stripe_rank=2)
    with pytest.raises(QuiverEngineError, match="num_stripes"):
        Engine.open(u8_index["dir"], "uint8", page_store="shared", num_stripes=3, stripe_rank=0)
    with Engine.open(u8_index["dir"], "uint8", page_store="shared", num_stripes=1, stripe_rank=0) as eng:
        h = eng.stripe_handle()
        assert len(h) == 64
        with pytest.raises(ValueError):
            eng.attach_stripes([h[:10]])
    with Engine.open(u8_index["dir"], "uint8") as eng:
        with pytest.raises(QuiverEngineError, match="not QV_PAGES_SHARED"):
            eng.stripe_handle()
