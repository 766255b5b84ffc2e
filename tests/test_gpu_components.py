"""Stage-level parity through the C ABI: LUT build + q'', ADC sums, exact L2.

Every value must be bit-identical to the oracle's restatement of the
reference (pq_device.cuh:9-36, kernel_helpers.cuh:271-286,
gpu_primitives.cuh:26-44).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fixture", ["u8_index", "f32_index", "odd_index"])
def test_lut_adc_l2_bit_exact(request, fixture):
    import torch
    from oracle import pyoracle
    from quiver_b200 import Engine, _build
    _build.build_engine()
    fx = request.getfixturevalue(fixture)
    ix = pyoracle.load_index(fx["dir"], fx["dtype"])
    q = fx["queries"][:16]
    nq, dim = q.shape
    M = ix.num_chunks
    with Engine.open(fx["dir"], fx["dtype"]) as eng:
        dq = torch.from_numpy(q).cuda()
        lut = torch.empty((nq, M, 256), dtype=torch.float32, device="cuda")
        q2 = torch.empty((nq, dim), dtype=torch.float32, device="cuda")
        eng.build_lut(dq, lut, q2)
        torch.cuda.synchronize()
        rng = np.random.default_rng(0)
        qof = np.repeat(np.arange(nq, dtype=np.int32), 64)
        ids = rng.integers(0, ix.num_points, size=qof.size).astype(np.int32)
        d_adc = torch.empty(qof.size, dtype=torch.float32, device="cuda")
        d_l2 = torch.empty(qof.size, dtype=torch.float32, device="cuda")
        eng.adc(lut, torch.from_numpy(qof).cuda(), torch.from_numpy(ids).cuda(), d_adc)
        eng.exact_l2(q2, torch.from_numpy(qof).cuda(), torch.from_numpy(ids).cuda(), d_l2)
        torch.cuda.synchronize()
        lut_h, q2_h = lut.cpu().numpy(), q2.cpu().numpy()
        adc_h, l2_h = d_adc.cpu().numpy(), d_l2.cpu().numpy()
    for i in range(nq):
        ref_lut, ref_q2 = pyoracle.build_lut(ix, q[i])
        np.testing.assert_array_equal(lut_h[i].view(np.uint32), ref_lut.view(np.uint32))
        np.testing.assert_array_equal(q2_h[i].view(np.uint32), ref_q2.view(np.uint32))
    for j in range(qof.size):
        ref_lut, ref_q2 = pyoracle.build_lut(ix, q[qof[j]])
        assert np.float32(adc_h[j]).view(np.uint32) == np.float32(pyoracle.adc(ref_lut, ix.codes[ids[j]])).view(np.uint32)
        assert np.float32(l2_h[j]).view(np.uint32) == np.float32(pyoracle.exact_l2(ix, ref_q2, int(ids[j]))).view(np.uint32)


@pytest.mark.parametrize("dtype,dim", [("uint8", 128), ("float", 96)])
def test_gpu_ground_truth_is_exact(dtype, dim):
    """The GPU brute force behind the benchmark's recall equals the exact host one."""
    from quiver_b200 import builder, workloads
    base = builder.synth_mixture(9, 300_000, dim, 30, 20.0 if dtype == "uint8" else 0.1, dtype)
    q = builder.synth_mixture(9, 64, dim, 30, 20.0 if dtype == "uint8" else 0.1, dtype, stream=1)
    ref, ref_d = builder.ground_truth(base, q, 10)
    got = workloads._gt_torch(base, q, 10, "cuda:0")
    exact = ((base[got].astype(np.float64) - q[:, None, :].astype(np.float64)) ** 2).sum(-1)
    if dtype == "uint8":  # integer distances: equal up to the choice among tied ids
        np.testing.assert_array_equal(np.sort(exact, axis=1), ref_d.astype(np.float64))
    else:  # fp32 GEMM vs double accumulation: the same set up to near-ties
        assert np.mean([len(set(a) & set(b)) for a, b in zip(got, ref)]) >= 9.9
