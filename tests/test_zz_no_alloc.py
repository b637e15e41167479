"""The allocation-free normalisation entry point against the allocating one.

``muzo_ns_normalize_noalloc`` serves callers that cannot allocate device memory (a runtime that
reserves the whole pool at start-up, a plugin inside another framework's allocator): its scratch
is a fixed device array inside the library. It must give the same normalised Newton-Schulz
inputs and flags as ``muzo_ns_prepare`` + ``muzo_ns_normalize`` with caller-provided scratch, on
two calls in a row (the second call must not see the first call's sums). This file is collected
last so that a run stopping at the first failure has run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch


def _lib():
    from muzo_clip_b200 import _lib

    return _lib


SHAPES = [(256, 512), (100, 37), (1024, 96)]


def _allocating(L, mats, device):
    """The existing path: caller-provided table, sums and flags."""
    outs = [torch.empty(m.shape, dtype=torch.bfloat16, device=device) for m in mats]
    segs, total = L.plan_linear([m.numel() for m in mats], [m.data_ptr() for m in mats], [o.data_ptr() for o in outs])
    table = L.to_device_table(segs, device)
    sums = torch.zeros((len(mats), L.NSUMS), dtype=torch.float64, device=device)
    flags = torch.zeros(len(mats), dtype=torch.int32, device=device)
    code = L.dtype_code(mats[0].dtype)
    L.launch("muzo_ns_prepare", table.data_ptr(), len(segs), total, code, sums.data_ptr(), flags.data_ptr(),
             L.stream_ptr(device))
    nsegs, ntot = L.plan_linear([m.numel() for m in mats], [o.data_ptr() for o in outs], [o.data_ptr() for o in outs])
    ntable = L.to_device_table(nsegs, device)
    L.launch("muzo_ns_normalize", ntable.data_ptr(), len(nsegs), ntot, sums.data_ptr(), flags.data_ptr(),
             L.stream_ptr(device))
    return outs, flags


def _noalloc(L, mats, device):
    outs = [torch.full(m.shape, 7.0, dtype=torch.bfloat16, device=device) for m in mats]
    flags = torch.full((len(mats),), -1, dtype=torch.int32, device=device)
    n = len(mats)
    ins = (ctypes.c_void_p * n)(*[m.data_ptr() for m in mats])
    ous = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
    numels = (ctypes.c_int64 * n)(*[m.numel() for m in mats])
    status = L.lib.muzo_ns_normalize_noalloc(ins, ous, numels, n, L.dtype_code(mats[0].dtype), flags.data_ptr(),
                                             L.stream_ptr(device))
    L.check(status, "muzo_ns_normalize_noalloc")
    return outs, flags


@pytest.mark.gpu
def test_noalloc_matches_allocating_path_on_consecutive_calls(device):
    L = _lib()
    g = torch.Generator(device="cpu").manual_seed(17)
    calls = [
        [torch.randn(s, generator=g).to(device) for s in SHAPES],                          # fp32
        [(torch.randn(s, generator=g) * 3).to(torch.bfloat16).to(device) for s in SHAPES],  # bf16
    ]
    calls[1][1].zero_()  # a zero matrix: flagged, as the reference returns zeros for it
    for mats in calls:
        want, want_flags = _allocating(L, mats, device)
        got, got_flags = _noalloc(L, mats, device)
        torch.cuda.synchronize()
        assert torch.equal(got_flags.cpu(), want_flags.cpu())
        for w, o in zip(want, got):
            # same arithmetic; the fp64 sums may differ in their last bits with atomic order,
            # which can move a quotient by one bf16 ulp
            diff = (w.float() - o.float()).abs()
            ulp = torch.clamp(w.float().abs(), min=2.0 ** -126) * 2.0 ** -7
            assert bool((diff <= ulp).all())
            assert (w == o).float().mean().item() >= 0.999


def test_noalloc_rejects_more_blocks_than_the_scratch_holds():
    L = _lib()
    n = 65
    arr = (ctypes.c_void_p * n)(*([16] * n))
    numels = (ctypes.c_int64 * n)(*([8] * n))
    assert L.lib.muzo_ns_normalize_noalloc(arr, arr, numels, n, 1, None, None) == 5  # MUZO_ERR_CAPACITY
