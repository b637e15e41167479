"""Deterministic parameter-wise noise on B200 (mirror of muzo_clip/prng.py).

``hash64_seed`` is the reference's host hash (prng.py:19-36), bit-exact. ``make_zo_noise_like``
(prng.py:39-81) writes the noise tensor with the library's fill kernel, which regenerates the
stream torch's CUDA generator yields for the same key: bit-exact for Rademacher noise and for the
Philox words under normal noise. Noise is produced on CUDA tensors only.
"""

from __future__ import annotations

import hashlib
from collections.abc import Iterator
from typing import Literal

import torch

from . import _lib

NoiseDistribution = Literal["normal", "rademacher"]


_MASK63 = (1 << 63) - 1


def hash64_seed(
    base_seed: int,
    param_name: str,
    param_shape: tuple[int, ...],
    block_index: int = 0,
) -> int:
    """Stable 63-bit key of one parameter block: blake2b-64 of "seed|name|d0,d1|block".

    The payload text and digest handling must equal the reference's byte for byte, because the
    key seeds the noise of every perturbation and of the momentum rebuild.
    """

    dims = ",".join(str(int(d)) for d in param_shape)
    text = f"{int(base_seed)}|{param_name}|{dims}|{int(block_index)}"
    digest = hashlib.blake2b(text.encode("utf-8"), digest_size=8).digest()
    return int.from_bytes(digest, "little") & _MASK63


def make_zo_noise_like(
    tensor: torch.Tensor,
    base_seed: int,
    param_name: str,
    block_index: int = 0,
    distribution: NoiseDistribution = "normal",
) -> torch.Tensor:
    """Deterministic ZO noise with the shape and dtype of ``tensor`` (CUDA tensors only)."""

    if not tensor.is_floating_point():
        raise TypeError("MuZO-Clip noise can only be generated for floating tensors")
    if distribution not in ("normal", "rademacher"):
        raise ValueError(f"Unsupported noise distribution: {distribution}")
    if tensor.device.type != "cuda":
        raise ValueError("muzo_clip_b200 generates noise on CUDA devices only")

    seed = hash64_seed(int(base_seed), param_name, tuple(tensor.shape), int(block_index))
    out = torch.empty(tensor.shape, dtype=tensor.dtype, device=tensor.device)
    if out.numel() == 0:
        return out
    dist = _lib.dist_code(distribution)
    sms, max_thr = _lib.device_geometry(tensor.device)
    segs, total = _lib.plan_segments([out.numel()], [0], [out.data_ptr()], dist, sms, max_thr)
    table = _lib.to_device_table(segs, tensor.device)
    _lib.launch("muzo_fill_noise", table.data_ptr(), len(segs), total, seed, dist,
                                 _lib.dtype_code(out.dtype), _lib.stream_ptr(tensor.device))
    return out


def iter_param_blocks(
    param: torch.Tensor,
    block_rows: int | None,
) -> Iterator[tuple[int, slice, torch.Tensor]]:
    """Row blocks of a 2-D parameter with their block index (prng.py:84-106).

    ``block_rows=None`` gives the whole matrix as block 0; otherwise consecutive chunks of
    ``block_rows`` rows numbered 0, 1, ... — the index feeds ``hash64_seed``.
    """

    if param.ndim != 2:
        raise ValueError("MuZO-Clip block iteration only supports 2D tensors")
    if block_rows is None:
        yield 0, slice(None), param
        return
    if block_rows <= 0:
        raise ValueError("block_rows must be positive or None")
    step = int(block_rows)
    total = int(param.shape[0])
    index = 0
    start = 0
    while start < total:
        rows = slice(start, min(total, start + step))
        yield index, rows, param[rows]
        index += 1
        start += step
