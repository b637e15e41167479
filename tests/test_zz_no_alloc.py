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


def _out_like(m, device, fill):
    """A bf16 output of m's shape; for a matrix without elements a view with a valid pointer."""
    if m.numel() == 0:
        return torch.empty(64, dtype=torch.bfloat16, device=device)[:0].view(m.shape)
    return torch.full(m.shape, fill, dtype=torch.bfloat16, device=device)


def _ptr(t):
    """A tensor's address; for one without elements (data_ptr() is 0) its storage's, which the
    entry point accepts as the pointer of an empty matrix."""
    return t.data_ptr() if t.numel() else t.untyped_storage().data_ptr()


def _allocating(L, mats, device):
    """The existing path: caller-provided table, sums and flags."""
    outs = [_out_like(m, device, 0.0) for m in mats]
    segs, total = L.plan_linear([m.numel() for m in mats], [_ptr(m) for m in mats], [_ptr(o) for o in outs])
    table = L.to_device_table(segs, device)
    sums = torch.zeros((len(mats), L.NSUMS), dtype=torch.float64, device=device)
    flags = torch.zeros(len(mats), dtype=torch.int32, device=device)
    code = L.dtype_code(mats[0].dtype)
    L.launch("muzo_ns_prepare", table.data_ptr(), len(segs), total, code, sums.data_ptr(), flags.data_ptr(),
             L.stream_ptr(device))
    nsegs, ntot = L.plan_linear([m.numel() for m in mats], [_ptr(o) for o in outs], [_ptr(o) for o in outs])
    ntable = L.to_device_table(nsegs, device)
    L.launch("muzo_ns_normalize", ntable.data_ptr(), len(nsegs), ntot, sums.data_ptr(), flags.data_ptr(),
             L.stream_ptr(device))
    return outs, flags


def _noalloc(L, mats, device):
    outs = [_out_like(m, device, 7.0) for m in mats]
    flags = torch.full((len(mats),), -1, dtype=torch.int32, device=device)
    n = len(mats)
    ins = (ctypes.c_void_p * n)(*[_ptr(m) for m in mats])
    ous = (ctypes.c_void_p * n)(*[_ptr(o) for o in outs])
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
        [(torch.randn(s, generator=g) * 3).to(torch.float16).to(device) for s in SHAPES],   # fp16
    ]
    calls[1][1].zero_()  # a zero matrix: flagged, as the reference returns zeros for it
    calls[2][0][3, 5] = float("inf")   # non-finite inputs: MUZO_FLAG_NONFINITE_INPUT
    calls[2][2][0, 0] = float("nan")
    # a matrix without elements among the others (a view with a valid base pointer)
    calls[0].insert(1, torch.empty(64, device=device)[:0].view(0, 4))
    for mats in calls:
        want, want_flags = _allocating(L, mats, device)
        got, got_flags = _noalloc(L, mats, device)
        torch.cuda.synchronize()
        assert torch.equal(got_flags.cpu(), want_flags.cpu())
        for w, o, m in zip(want, got, mats):
            if not torch.isfinite(m).all():
                continue   # flagged: the step skips the matrix, its normalised values are not used
            # same arithmetic; the fp64 sums may differ in their last bits with atomic order,
            # which can move a quotient by one bf16 ulp
            diff = (w.float() - o.float()).abs()
            ulp = torch.clamp(w.float().abs(), min=2.0 ** -126) * 2.0 ** -7
            assert bool((diff <= ulp).all())
            if w.numel():
                assert (w == o).float().mean().item() >= 0.999
    # the flags themselves: the non-finite fp16 matrices and the zero bf16 matrix
    flags = [_noalloc(L, mats, device)[1].cpu().tolist() for mats in calls]
    assert flags[2][0] & 1 and flags[2][2] & 1 and not flags[2][1] & 1   # MUZO_FLAG_NONFINITE_INPUT
    assert flags[1][1] != 0


def test_noalloc_rejects_more_blocks_than_the_scratch_holds():
    L = _lib()
    n = 65
    arr = (ctypes.c_void_p * n)(*([16] * n))
    numels = (ctypes.c_int64 * n)(*([8] * n))
    assert L.lib.muzo_ns_normalize_noalloc(arr, arr, numels, n, 1, None, None) == 5  # MUZO_ERR_CAPACITY
