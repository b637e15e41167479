"""ctypes binding of ``libmuzo_b200.so`` (the C ABI declared in ``include/muzo_b200.h``).

The library is the only compute path of this package: if it is missing or fails to load, the
import of this module raises and nothing falls back to PyTorch or the CPU.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np
import torch

_LIB_PATH = Path(os.environ.get("MUZO_B200_LIB", Path(__file__).with_name("libmuzo_b200.so")))

if not _LIB_PATH.exists():
    raise ImportError(
        f"muzo_clip_b200: native library {_LIB_PATH} not found; build it with "
        "`python muzo-clip_b200/build.py` (nvcc, sm_100a)"
    )

lib = ctypes.CDLL(str(_LIB_PATH))

# ---------------------------------------------------------------- ABI constants
OK = 0
ERR_ARG, ERR_DTYPE, ERR_ALIGN, ERR_CUDA, ERR_CAPACITY, ERR_UNSUPPORTED = 1, 2, 3, 4, 5, 6
F32, BF16, F16 = 0, 1, 2
NORMAL, RADEMACHER = 0, 1
EPI_STORE, EPI_POLY, EPI_UPDATE = 0, 1, 2
ITEMS_PER_CTA = 1024
IPC_HANDLE_BYTES = 64
NSUMS = 8
SUM_M2, SUM_X2, SUM_W2, SUM_U2, SUM_U2_CLIPPED = 0, 1, 2, 3, 4
FLAG_NONFINITE_INPUT, FLAG_ZERO_NORM, FLAG_NONFINITE_OUTPUT = 1, 2, 4
NSTATS = 4
STAT_RATIO_BEFORE, STAT_CLIP_FACTOR, STAT_ZEROED = 0, 1, 2

SEGMENT_DTYPE = np.dtype(
    [
        ("param", np.uint64),
        ("out", np.uint64),
        ("numel", np.int64),
        ("item_begin", np.int64),
        ("philox_offset", np.uint64),
        ("threads", np.uint32),
        ("block_index", np.int32),
        ("elem_start", np.int64),
        ("kept", np.uint64),
    ]
)
assert SEGMENT_DTYPE.itemsize == 64

_c = ctypes
_vp = _c.c_void_p
_i64 = _c.c_int64
_u64 = _c.c_uint64
_i32 = _c.c_int
_f32 = _c.c_float
_f64 = _c.c_double

_SIGNATURES = {
    "muzo_abi_version": ([], _i32),
    "muzo_status_string": ([_i32], _c.c_char_p),
    "muzo_last_cuda_error": ([], _i32),
    "muzo_hash64_seed": ([_u64, _c.c_char_p, _vp, _i32, _i64, _vp], _i32),
    "muzo_plan_segments": ([_vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _i32, _vp, _vp], _i32),
    "muzo_plan_linear": ([_vp, _vp, _vp, _i32, _vp, _i32, _vp, _vp], _i32),
    "muzo_fill_noise": ([_vp, _i32, _i64, _u64, _i32, _i32, _vp], _i32),
    "muzo_perturb_segments": ([_vp, _i32, _i64, _vp, _i32, _i32, _f32, _vp], _i32),
    "muzo_perturb_segments_keep_noise": ([_vp, _i32, _i64, _vp, _i32, _f32, _vp], _i32),
    "muzo_perturb_kept_noise": ([_vp, _i32, _i64, _i32, _f32, _vp], _i32),
    "muzo_rebuild_segments": (
        [_vp, _i32, _i64, _vp, _vp, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _i32, _vp],
        _i32,
    ),
    "muzo_rebuild_segments_kept": (
        [_vp, _i32, _i64, _vp, _vp, _i32, _i32, _i32, _f32, _vp, _vp, _i32, _vp],
        _i32,
    ),
    "muzo_rebuild_segments_history": (
        [_vp, _i32, _i64, _vp, _vp, _vp, _i32, _i32, _i32, _f32, _vp, _vp, _i32, _vp],
        _i32,
    ),
    "muzo_rebuild_kept_linear": ([_vp, _i32, _i64, _vp, _vp, _i32, _i32, _i32, _f32, _vp, _vp, _vp], _i32),
    "muzo_ns_prepare": ([_vp, _i32, _i64, _i32, _vp, _vp, _vp], _i32),
    "muzo_ns_normalize": ([_vp, _i32, _i64, _vp, _vp, _vp], _i32),
    "muzo_ns_gemm": (
        [_vp, _i64, _i64, _i32, _vp, _i64, _i64, _i32, _vp, _i64, _i64, _vp, _i32, _f32, _f32,
         _i64, _i64, _i64, _i64, _i32, _vp, _vp, _vp, _vp, _vp],
        _i32,
    ),
    "muzo_update_sumsq": ([_vp, _i32, _i64, _vp, _vp, _vp, _vp], _i32),
    "muzo_apply_update": (
        [_vp, _i32, _i64, _i32, _vp, _f32, _f64, _i32, _f32, _vp, _vp, _vp, _vp],
        _i32,
    ),
    "muzo_qk_scale_rows": ([_vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp], _i32),
    "muzo_qk_max": (
        [_vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _f32, _vp,
         _vp, _vp],
        _i32,
    ),
    "muzo_qk_max_ranges": (
        [_vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _vp, _vp,
         _f32, _vp, _vp, _vp],
        _i32,
    ),
    "muzo_logits_head_max": ([_vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp], _i32),
    "muzo_max_merge": ([_vp, _vp, _vp, _i64, _vp], _i32),
    "muzo_ns_normalize_noalloc": ([_vp, _vp, _vp, _i32, _i32, _vp, _vp], _i32),
    "muzo_attention_max": (
        [_vp, _vp, _vp, _vp, _i32] + [_i64] * 6 + [_i64] * 12 + [_i32, _f32, _vp, _vp, _vp, _vp, _vp, _vp],
        _i32,
    ),
    "muzo_ipc_export": ([_vp, _vp, _vp, _vp], _i32),
    "muzo_ipc_import": ([_vp, _vp], _i32),
    "muzo_ipc_close": ([_vp], _i32),
    "muzo_push_blocks": ([_vp, _vp, _vp, _i32, _vp], _i32),
}

for _name, (_args, _ret) in _SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = _args
    _fn.restype = _ret

EXPORTED = tuple(_SIGNATURES)


class MuzoError(RuntimeError):
    """A native entry point returned a non-zero status."""


# Kernels each compute entry point enqueues (for launch accounting by benchmarks).
KERNELS_PER_CALL = {
    "muzo_fill_noise": 1, "muzo_perturb_segments": 1, "muzo_perturb_segments_keep_noise": 1,
    "muzo_perturb_kept_noise": 1, "muzo_rebuild_segments": 1, "muzo_rebuild_segments_kept": 1,
    "muzo_ns_prepare": 1, "muzo_rebuild_segments_history": 1, "muzo_rebuild_kept_linear": 1,
    "muzo_ns_normalize": 1, "muzo_ns_gemm": 1, "muzo_update_sumsq": 1, "muzo_apply_update": 1,
    "muzo_qk_scale_rows": 1, "muzo_qk_max": 3, "muzo_qk_max_ranges": 3, "muzo_logits_head_max": 3, "muzo_max_merge": 1,
    "muzo_ns_normalize_noalloc": 3, "muzo_attention_max": 3, "muzo_ipc_export": 0, "muzo_ipc_import": 0, "muzo_ipc_close": 0,
    "muzo_push_blocks": 0,
}
launch_count = 0


def launch(name: str, *args) -> None:
    """Call a compute entry point, count its kernels and raise on a non-zero status."""
    global launch_count
    status = getattr(lib, name)(*args)
    check(status, name)
    launch_count += KERNELS_PER_CALL.get(name, 1)


def check(status: int, what: str) -> None:
    if status != OK:
        msg = lib.muzo_status_string(status).decode()
        if status == ERR_CUDA:
            msg += f" (cudaError {lib.muzo_last_cuda_error()})"
        raise MuzoError(f"{what}: {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float16:
        return F16
    if dtype == torch.float32:
        return F32
    raise TypeError(f"muzo_clip_b200 kernels support float32, bfloat16 and float16, not {dtype}")


def dist_code(distribution: str) -> int:
    if distribution == "normal":
        return NORMAL
    if distribution == "rademacher":
        return RADEMACHER
    raise ValueError(f"Unsupported noise distribution: {distribution}")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_DEVICE_PROPS: dict[int, tuple[int, int]] = {}


def device_geometry(device: torch.device) -> tuple[int, int]:
    """(multiProcessorCount, maxThreadsPerMultiProcessor) — the values torch's generator uses."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _DEVICE_PROPS:
        p = torch.cuda.get_device_properties(idx)
        _DEVICE_PROPS[idx] = (int(p.multi_processor_count), int(p.max_threads_per_multi_processor))
    return _DEVICE_PROPS[idx]


def plan_segments(numels, params, outs, dist: int, sm_count: int, max_threads: int) -> tuple[np.ndarray, int]:
    """Host planning of noise launch units. Returns (segments, total_items)."""
    n = len(numels)
    numel_arr = np.asarray(numels, dtype=np.int64)
    param_arr = np.asarray([int(p) for p in params], dtype=np.uint64)
    out_arr = np.asarray([int(o) for o in outs], dtype=np.uint64) if outs is not None else None
    cap = 4 * max(n, 1) + 16
    while True:
        segs = np.zeros(cap, dtype=SEGMENT_DTYPE)
        nsegs = _c.c_int(0)
        total = _c.c_int64(0)
        st = lib.muzo_plan_segments(
            numel_arr.ctypes.data, param_arr.ctypes.data,
            out_arr.ctypes.data if out_arr is not None else None, n, dist, sm_count, max_threads,
            segs.ctypes.data, cap, _c.byref(nsegs), _c.byref(total),
        )
        if st == ERR_CAPACITY:
            cap *= 2
            continue
        check(st, "muzo_plan_segments")
        return segs[: nsegs.value].copy(), int(total.value)


def plan_linear(numels, params, outs) -> tuple[np.ndarray, int]:
    n = len(numels)
    numel_arr = np.asarray(numels, dtype=np.int64)
    param_arr = np.asarray([int(p) for p in params], dtype=np.uint64)
    out_arr = np.asarray([int(o) for o in outs], dtype=np.uint64) if outs is not None else None
    segs = np.zeros(max(n, 1), dtype=SEGMENT_DTYPE)
    nsegs = _c.c_int(0)
    total = _c.c_int64(0)
    st = lib.muzo_plan_linear(
        numel_arr.ctypes.data, param_arr.ctypes.data,
        out_arr.ctypes.data if out_arr is not None else None, n, segs.ctypes.data, n,
        _c.byref(nsegs), _c.byref(total),
    )
    check(st, "muzo_plan_linear")
    return segs[: nsegs.value].copy(), int(total.value)


def to_device_table(segs: np.ndarray, device: torch.device) -> torch.Tensor:
    """Copy a segment table to device memory (stream-ordered on the current stream)."""
    host = torch.from_numpy(segs.view(np.uint8).copy())
    return host.to(device=device, non_blocking=False)


def hash64_seed_native(base_seed: int, name: str, shape, block_index: int) -> int:
    dims = np.asarray([int(d) for d in shape], dtype=np.int64)
    out = _c.c_uint64(0)
    check(
        lib.muzo_hash64_seed(int(base_seed) & 0xFFFFFFFFFFFFFFFF, name.encode("utf-8"),
                             dims.ctypes.data if dims.size else None, int(dims.size), int(block_index),
                             _c.byref(out)),
        "muzo_hash64_seed",
    )
    return int(out.value)
