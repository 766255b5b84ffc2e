"""Batched ADC (``qv_adc_batch``): both kernels against the oracle's chunk-ordered fp32 sum.

The sum must be bit-identical to the sequential loop of
src/shared/kernel_helpers.cuh:271-286 for every pair; ids outside
``[0, num_points)`` give NaN.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest


def _luts(rng, nq, M):
    # LUT values of the size and spread squared-distance tables have, plus exact zeros.
    lut = (rng.random((nq, M, 256), dtype=np.float32) * 4096.0).astype(np.float32)
    lut[:, :, 7] = 0.0
    return lut


def _same(got, ref):
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(ref))
    ok = ~np.isnan(ref)
    np.testing.assert_array_equal(got[ok].view(np.uint32), ref[ok].view(np.uint32))


def test_oracle_adc_batch_equals_scalar_oracle():
    """The vectorised restatement equals the C oracle's scalar loop pair by pair."""
    from oracle import pyoracle
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 256, size=(500, 32), dtype=np.uint8)
    luts = _luts(rng, 3, 32)
    ids = rng.integers(-5, 505, size=(3, 40))
    got = pyoracle.adc_batch(luts, codes, ids)
    for q in range(3):
        for i in range(40):
            v = ids[q, i]
            if 0 <= v < 500:
                assert got[q, i].view(np.uint32) == np.float32(pyoracle.adc(luts[q], codes[v])).view(np.uint32)
            else:
                assert np.isnan(got[q, i])


def test_adc_batch_argument_checks_without_gpu():
    """Argument validation in the C ABI runs before any device call."""
    from quiver_b200 import _lib
    lib = _lib.engine_lib()
    assert lib.qv_adc_batch(None, 10, 32, None, 0, None, None, 5, None, 0, None) == _lib.QV_OK  # nq == 0
    assert lib.qv_adc_batch(None, 10, 200, None, 1, None, None, 5, None, 0, None) == 1
    assert b"M must be" in lib.qv_last_error()
    assert lib.qv_adc_batch(None, 10, 32, None, 1, None, None, 5, None, 9, None) == 1
    assert lib.qv_adc_batch(None, 10, 32, None, 1, None, None, 5, None, 0, None) == 1
    assert b"required" in lib.qv_last_error()
    assert lib.qv_adc_batch(C.c_void_p(16), 10, 32, C.c_void_p(20), 1, C.c_void_p(16), None, 5, C.c_void_p(16),
                            0, None) == 1  # luts not 16-byte aligned
    assert b"aligned" in lib.qv_last_error()
    assert lib.qv_adc_batch(C.c_void_p(16), 10, 33, C.c_void_p(32), 1, C.c_void_p(16), None, 5, C.c_void_p(16),
                            0, None) == 1  # M not a multiple of 4
    assert b"multiple of 4" in lib.qv_last_error()


def _gpu_case(seed, num_points, M, nq, n, invalid=True):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 256, size=(num_points, M), dtype=np.uint8)
    luts = _luts(rng, nq, M)
    ids = rng.integers(0, num_points, size=(nq, n)).astype(np.int32)
    if invalid and n >= 4:
        ids[0, :3] = [-1, num_points, np.iinfo(np.int32).max]
        ids[-1, -1] = np.iinfo(np.int32).min
    return codes, luts, ids


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", ["thread", "pipe", "auto"])
@pytest.mark.parametrize("nq,n", [(5, 10000), (3, 9999), (2, 31), (1, 1), (3, 100_003)])
def test_adc_batch_ids_bit_exact(kernel, nq, n):
    import torch
    from oracle import pyoracle
    from quiver_b200.adc import adc_batch
    codes, luts, ids = _gpu_case(11 + n, 70_001, 32, nq, n)
    got = adc_batch(torch.from_numpy(codes).cuda(), torch.from_numpy(luts).cuda(), torch.from_numpy(ids).cuda(),
                    kernel=kernel)
    torch.cuda.synchronize()
    _same(got.cpu().numpy(), pyoracle.adc_batch(luts, codes, ids))


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", ["thread", "pipe"])
def test_adc_batch_ranges_bit_exact(kernel):
    """Contiguous ranges, including ones that start before 0 or run past the last code (NaN there)."""
    import torch
    from oracle import pyoracle
    from quiver_b200.adc import adc_batch
    num_points, n = 50_000, 12_345
    codes, luts, _ = _gpu_case(5, num_points, 32, 4, 1, invalid=False)
    first = np.array([0, 1234, num_points - 5000, -7], dtype=np.int64)
    got = adc_batch(torch.from_numpy(codes).cuda(), torch.from_numpy(luts).cuda(), first=torch.from_numpy(first).cuda(),
                    n_per_query=n, kernel=kernel)
    torch.cuda.synchronize()
    ids = first[:, None] + np.arange(n)[None, :]
    _same(got.cpu().numpy(), pyoracle.adc_batch(luts, codes, ids))


@pytest.mark.gpu
@pytest.mark.parametrize("M", [8, 16, 64, 128])
def test_adc_batch_other_widths(M):
    """Widths other than 32 bytes take the byte-loading thread kernel."""
    import torch
    from oracle import pyoracle
    from quiver_b200 import QuiverEngineError
    from quiver_b200.adc import adc_batch
    codes, luts, ids = _gpu_case(M, 20_000, M, 3, 5000)
    dc, dl, di = torch.from_numpy(codes).cuda(), torch.from_numpy(luts).cuda(), torch.from_numpy(ids).cuda()
    got = adc_batch(dc, dl, di)
    torch.cuda.synchronize()
    _same(got.cpu().numpy(), pyoracle.adc_batch(luts, codes, ids))
    with pytest.raises(QuiverEngineError, match="pipe kernel"):
        adc_batch(dc, dl, di, kernel="pipe")


@pytest.mark.gpu
def test_adc_batch_unaligned_codes():
    """Codes that do not start on a 16-byte boundary: byte loads, same sums; the pipe kernel refuses."""
    import torch
    from oracle import pyoracle
    from quiver_b200 import QuiverEngineError
    from quiver_b200.adc import adc_batch
    codes, luts, ids = _gpu_case(8, 30_000, 32, 2, 9000)
    flat = torch.zeros(codes.size + 4, dtype=torch.uint8, device="cuda")
    flat[4:] = torch.from_numpy(codes.reshape(-1)).cuda()
    dc = flat[4:].view(codes.shape)
    assert dc.data_ptr() % 16 == 4
    got = adc_batch(dc, torch.from_numpy(luts).cuda(), torch.from_numpy(ids).cuda())
    torch.cuda.synchronize()
    _same(got.cpu().numpy(), pyoracle.adc_batch(luts, codes, ids))
    with pytest.raises(QuiverEngineError, match="pipe kernel"):
        adc_batch(dc, torch.from_numpy(luts).cuda(), torch.from_numpy(ids).cuda(), kernel="pipe")


@pytest.mark.gpu
def test_adc_batch_kernels_agree_at_scale():
    """Larger than L2: both kernels give the same bits for every pair, and a sample matches the oracle."""
    import torch
    from oracle import pyoracle
    from quiver_b200.adc import adc_batch
    num_points, nq, n = 8_000_000, 64, 65_536
    g = torch.Generator(device="cuda").manual_seed(1)
    codes = torch.randint(0, 256, (num_points, 32), dtype=torch.uint8, device="cuda", generator=g)
    luts = torch.rand((nq, 32, 256), device="cuda", generator=g) * 4096.0
    ids = torch.randint(0, num_points, (nq, n), dtype=torch.int32, device="cuda", generator=g)
    a = adc_batch(codes, luts, ids, kernel="pipe")
    b = adc_batch(codes, luts, ids, kernel="thread")
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    rows = ids[:, :: 997].cpu().numpy()
    ref = pyoracle.adc_batch(luts.cpu().numpy(), codes.cpu().numpy(), rows)
    _same(a[:, :: 997].cpu().numpy(), ref)
