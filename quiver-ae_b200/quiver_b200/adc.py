"""Batched PQ asymmetric distances on CUDA tensors (``qv_adc_batch``).

Query ``q`` scores ``n`` codes with its LUT ``luts[q]`` (``[M, 256]`` fp32,
the table ``PQSearchData::init_query`` builds, src/shared/index/pq_device.cuh:9-36);
each distance is the chunk-ordered fp32 sum the search's scoring loop computes
(src/shared/kernel_helpers.cuh:271-286).  The codes are either gathered by id
(``ids[q, i]``, the search's access pattern) or read as a contiguous range
``first[q] .. first[q] + n``.  An id outside ``[0, num_points)`` gives NaN.
"""
from __future__ import annotations

import ctypes as C

from . import _lib
from .engine import _check

KERNELS = {"auto": _lib.QV_ADC_AUTO, "thread": _lib.QV_ADC_THREAD, "pipe": _lib.QV_ADC_PIPE}


def adc_batch(codes, luts, ids=None, first=None, n_per_query: int | None = None, out=None,
              kernel: str = "auto", stream=None):
    """Return ``out[q, i]`` = ADC distance of query ``q`` to its ``i``-th code.

    codes: uint8 ``[num_points, M]``; luts: float32 ``[nq, M, 256]`` (or
    ``[nq, M * 256]``); ids: int32 ``[nq, n]``, or None with ``first``: int64
    ``[nq]`` and ``n_per_query``.  All on one CUDA device; asynchronous on
    ``stream`` (default: torch's current stream).
    """
    import torch
    if codes.dtype != torch.uint8 or codes.dim() != 2 or not codes.is_cuda:
        raise ValueError("codes must be a CUDA uint8 tensor [num_points, M]")
    num_points, M = codes.shape
    nq = luts.shape[0]
    if luts.dtype != torch.float32 or luts.numel() != nq * M * 256 or luts.device != codes.device:
        raise ValueError(f"luts must be float32 [nq, {M}, 256] on the codes' device")
    if ids is not None:
        if ids.dtype != torch.int32 or ids.dim() != 2 or ids.shape[0] != nq or ids.device != codes.device:
            raise ValueError("ids must be int32 [nq, n] on the codes' device")
        n = ids.shape[1]
        ids = ids.contiguous()
        first_ptr = None
    else:
        if first is None or n_per_query is None:
            raise ValueError("give ids, or first and n_per_query")
        if first.dtype != torch.int64 or first.numel() != nq or first.device != codes.device:
            raise ValueError("first must be int64 [nq] on the codes' device")
        n = int(n_per_query)
        first = first.contiguous()
        first_ptr = C.c_void_p(first.data_ptr())
    if kernel not in KERNELS:
        raise ValueError(f"kernel must be one of {sorted(KERNELS)}")
    codes = codes.contiguous()
    luts = luts.contiguous()
    if out is None:
        out = torch.empty((nq, n), dtype=torch.float32, device=codes.device)
    elif (out.dtype != torch.float32 or out.numel() != nq * n or not out.is_contiguous()
          or out.device != codes.device):
        raise ValueError("out must be a contiguous float32 tensor of nq * n elements on the codes' device")
    st = stream if stream is not None else torch.cuda.current_stream(codes.device)
    if stream is not None:
        # the inputs (or their contiguous copies) stay allocated until the kernel on `stream` has read them
        for t in (codes, luts, ids, first, out):
            if t is not None:
                t.record_stream(stream)
    with torch.cuda.device(codes.device):  # the launch goes to the current device
        _check(_lib.engine_lib().qv_adc_batch(
            C.c_void_p(codes.data_ptr()), num_points, M, C.c_void_p(luts.data_ptr()), nq,
            C.c_void_p(ids.data_ptr()) if ids is not None else None, first_ptr, n,
            C.c_void_p(out.data_ptr()), KERNELS[kernel], C.c_void_p(st.cuda_stream)))
    return out
