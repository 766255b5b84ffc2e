"""Striped page store: page p on stripe p mod S of S devices' HBM.

For indexes whose graph pages exceed one GPU's HBM (configs 3 and 4 of the
hot-path scope), pages are striped page-wise across GPUs and the search GPU
reads other GPUs' stripes with peer loads over NVLink.  On one GPU the same
code runs with every stripe on the search device (separate allocations), so
the addressing is checked anywhere; with two GPUs visible the stripes are
also placed on the peer.  Results must equal the unstriped store's bit for
bit.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _search(eng, fx, **kw):
    from quiver_b200 import SearchParams
    ids, dists, found = eng.search(fx["queries"], SearchParams(early_exit_policy="none", **kw))
    return ids, dists


@pytest.fixture(scope="module")
def plain(u8_index):
    from quiver_b200 import Engine
    with Engine.open(u8_index["dir"], "uint8") as eng:
        yield {(W, q): _search(eng, u8_index, topk=10, ef_search=48, pipe_width=W, queries_per_block=q)
               for W in (1, 2) for q in (1, 2)}


@pytest.mark.parametrize("stripes", [[0], [0, 0], [0, 0, 0, 0]])
def test_striped_on_one_device_equals_plain(u8_index, plain, stripes):
    from quiver_b200 import Engine
    with Engine.open(u8_index["dir"], "uint8", page_store="striped", stripe_devices=stripes) as eng:
        for (W, q), (ids, dists) in plain.items():
            got = _search(eng, u8_index, topk=10, ef_search=48, pipe_width=W, queries_per_block=q)
            np.testing.assert_array_equal(got[0], ids)
            np.testing.assert_array_equal(got[1].view(np.uint32), dists.view(np.uint32))


def test_striped_exact_l2_component(u8_index):
    """The exact-L2 component kernel reads records through the same addressing."""
    import torch
    from quiver_b200 import Engine
    q2 = torch.tensor(u8_index["queries"][:4], device="cuda")
    ids = torch.arange(0, 6000, 37, dtype=torch.int32, device="cuda")
    qof = (torch.arange(ids.numel(), device="cuda") % 4).to(torch.int32)
    outs = []
    for kw in ({}, {"page_store": "striped", "stripe_devices": [0, 0, 0, 0, 0, 0, 0, 0]}):
        with Engine.open(u8_index["dir"], "uint8", **kw) as eng:
            out = torch.empty(ids.numel(), dtype=torch.float32, device="cuda")
            eng.exact_l2(q2, qof, ids, out)
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
    np.testing.assert_array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_striped_bad_arguments(u8_index):
    from quiver_b200 import Engine, QuiverEngineError
    with pytest.raises(QuiverEngineError, match="num_stripes"):
        Engine.open(u8_index["dir"], "uint8", page_store="striped", stripe_devices=[0, 0, 0])
    with pytest.raises(QuiverEngineError, match="out of range"):
        Engine.open(u8_index["dir"], "uint8", page_store="striped", stripe_devices=[0, 64])


def test_striped_across_two_gpus(u8_index, plain):
    """Half the pages on the peer GPU, read over NVLink."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from quiver_b200 import Engine
    with Engine.open(u8_index["dir"], "uint8", page_store="striped", stripe_devices=[0, 1]) as eng:
        for (W, q), (ids, dists) in plain.items():
            got = _search(eng, u8_index, topk=10, ef_search=48, pipe_width=W, queries_per_block=q)
            np.testing.assert_array_equal(got[0], ids)
            np.testing.assert_array_equal(got[1].view(np.uint32), dists.view(np.uint32))
