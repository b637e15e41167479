"""Device helpers of QK-Clip: per-head max-logit kernels, the probe attention function that
transformers calls during a probe forward, and the q/k row scaling."""

from __future__ import annotations

import contextvars
import os
import weakref

import numpy as np
import torch

from . import _lib

_ACTIVE = contextvars.ContextVar("muzo_qk_controller", default=None)
_REGISTERED = False


def set_active_controller(ctrl):
    return _ACTIVE.set(ctrl)


def reset_active_controller(token) -> None:
    _ACTIVE.reset(token)


# ---------------------------------------------------------------- reductions


def _check_cuda(t: torch.Tensor) -> None:
    if t.device.type != "cuda":
        raise ValueError("muzo_clip_b200 QK-Clip kernels run on CUDA tensors only")


def logits_head_max(logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-head max over [B, H, Sq, Sk] logits and a validity word (0 when any logit is
    non-finite), both on the device."""
    _check_cuda(logits)
    b, h, sq, sk = (int(v) for v in logits.shape)
    out = torch.empty(h, dtype=torch.float32, device=logits.device)
    valid = torch.empty(1, dtype=torch.int32, device=logits.device)
    sb, sh, sqs, sks = (int(v) for v in logits.stride())
    _lib.launch("muzo_logits_head_max", logits.data_ptr(), _lib.dtype_code(logits.dtype), b, h, sq, sk, sb, sh, sqs,
                                      sks, out.data_ptr(), valid.data_ptr(), _lib.stream_ptr(logits.device))
    return out, valid


def qk_head_max(query: torch.Tensor, key: torch.Tensor, scaling: float, causal: bool,
                attention_mask: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-head max of the eager pre-softmax logits of one attention call, from Q [B, Hq, Sq, D]
    and K [B, Hkv, Sk, D] (any strides with D contiguous). A padding mask (per batch row a
    contiguous range of visible keys, with or without causality) runs on the same kernels with
    per-batch key ranges; any other mask reduces explicit logits."""
    _check_cuda(query)
    key_lo = key_hi = None
    ranges = None
    if attention_mask is not None:
        ranges = mask_key_ranges(attention_mask, query.shape[0], query.shape[2], key.shape[2])
    if attention_mask is not None and ranges is None:
        # a mask that is not a padding mask (e.g. block-diagonal or per-head): reduce explicit logits
        group = query.shape[1] // key.shape[1]
        kr = key.repeat_interleave(group, dim=1)
        if attention_mask.dtype == torch.bool:
            attention_mask = eager_additive_mask(attention_mask, causal, query.dtype)
        logits = torch.matmul(query, kr.transpose(2, 3)) * scaling + attention_mask
        return logits_head_max(logits)
    if ranges is not None:
        causal, key_lo, key_hi = ranges
    q, k = query, key
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    b, hq, sq, d = (int(v) for v in q.shape)
    hkv, sk = int(k.shape[1]), int(k.shape[2])
    out = torch.empty(hq, dtype=torch.float32, device=q.device)
    valid = torch.empty(1, dtype=torch.int32, device=q.device)
    _lib.launch("muzo_qk_max_ranges", q.data_ptr(), k.data_ptr(), _lib.dtype_code(q.dtype), b, hq, hkv, sq, sk, d,
                q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), 1 if causal else 0,
                key_lo.data_ptr() if key_lo is not None else None, key_hi.data_ptr() if key_hi is not None else None,
                float(scaling), out.data_ptr(), valid.data_ptr(), _lib.stream_ptr(q.device))
    return out, valid


def eager_additive_mask(keep: torch.Tensor, causal: bool, dtype: torch.dtype) -> torch.Tensor:
    """SDPA's boolean mask (True = attend) in eager attention's additive form (0 or the dtype's
    minimum). transformers un-masks rows that would be fully masked (padding queries) so that SDPA
    returns no NaN; eager attention keeps them masked. In a causal model such a row is the one
    that sees a key above the (end-aligned) diagonal, and it is masked again here."""
    if causal:
        sq, sk = keep.shape[-2], keep.shape[-1]
        i = torch.arange(sq, device=keep.device)[:, None] + (sk - sq)
        above = torch.arange(sk, device=keep.device)[None, :] > i
        keep = keep & ~(keep & above).any(dim=-1, keepdim=True)
    return torch.zeros(keep.shape, dtype=dtype, device=keep.device).masked_fill(~keep, torch.finfo(dtype).min)


# mask object id -> (weak reference, (batch, sq, sk, version), result): transformers builds one
# mask per forward and hands the same tensor to every layer, so the classification (one host
# sync) runs once per forward instead of once per layer
_RANGES_CACHE: dict[int, tuple] = {}


def mask_key_ranges(mask: torch.Tensor, batch: int, sq: int, sk: int):
    """Classify a [B|1, 1, Sq, Sk] attention mask (boolean, True = attend, or additive: 0 or at
    most half the dtype's minimum). Returns (causal, key_lo, key_hi) when every batch row b
    attends exactly to the keys [lo_b, hi_b) — and, when causal, only to those at or below the
    end-aligned diagonal — with key_lo / key_hi int32 device tensors [batch], or both None when
    every row sees all keys (no padding); None for any other mask. A query row that sees no key
    under the causal pattern may attend everywhere in a boolean mask (transformers lets such
    padding rows attend so that SDPA returns no NaN): eager attention masks it, and so does this
    classification. Cached per mask tensor and version."""
    try:
        key = (int(batch), int(sq), int(sk), mask._version)
    except RuntimeError:  # inference tensors track no version: no caching
        return _key_ranges_uncached(mask, batch, sq, sk)
    entry = _RANGES_CACHE.get(id(mask))
    if entry is not None and entry[0]() is mask and entry[1] == key:
        return entry[2]
    result = _key_ranges_uncached(mask, batch, sq, sk)
    if len(_RANGES_CACHE) >= 64:
        _RANGES_CACHE.clear()
    _RANGES_CACHE[id(mask)] = (weakref.ref(mask), key, result)
    return result


def _key_ranges_uncached(mask: torch.Tensor, batch: int, sq: int, sk: int):
    if mask.ndim != 4 or mask.shape[1] != 1 or mask.shape[-2] != sq or mask.shape[-1] != sk:
        return None
    if mask.shape[0] not in (1, batch) or sq == 0 or sk == 0:
        return None
    dev = mask.device
    if mask.dtype == torch.bool:
        keep = mask[:, 0]
        binary = torch.ones((), dtype=torch.bool, device=dev)
    elif mask.is_floating_point():
        m = mask[:, 0]
        keep = m == 0
        binary = (keep | (m <= torch.finfo(m.dtype).min / 2)).all()
    else:
        return None
    j = torch.arange(sk, device=dev)
    # the last query row sees the whole range under both patterns (never a padding row without
    # keys, which a boolean mask may have let attend everywhere)
    seen = keep[:, -1, :]                                             # [B', Sk]
    lo = torch.where(seen, j, sk).amin(dim=-1)                        # Sk when the row sees nothing
    hi = torch.where(seen, j + 1, 0).amax(dim=-1)
    in_range = (j >= lo[:, None]) & (j < hi[:, None])                 # [B', Sk]
    lower = j[None, :] <= torch.arange(sq, device=dev)[:, None] + (sk - sq)   # [Sq, Sk]
    want_c = lower[None] & in_range[:, None, :]
    unmasked = keep.all(dim=-1, keepdim=True) & ~want_c.any(dim=-1, keepdim=True)
    causal_ok = ((keep == want_c) | unmasked).all()
    full_ok = (keep == in_range[:, None, :]).all()
    flags = torch.stack([binary, causal_ok, full_ok]).to(torch.int64)
    padded = ((lo != 0) | (hi != sk)).any().to(torch.int64)[None]
    binary, causal_ok, full_ok, any_pad = (bool(v) for v in torch.cat([flags, padded]).tolist())
    if not binary or not (causal_ok or full_ok):
        return None
    if not any_pad:
        return causal_ok, None, None
    lo = lo.to(torch.int32).expand(batch).contiguous()
    hi = hi.to(torch.int32).expand(batch).contiguous()
    return causal_ok, lo, hi


def _is_plain_causal(mask: torch.Tensor, sq: int, sk: int) -> bool:
    """True when a [B|1, 1, Sq, Sk] mask is the plain causal mask for every batch row."""
    r = mask_key_ranges(mask, mask.shape[0] if mask.ndim == 4 else 1, sq, sk)
    return r is not None and r[0] and r[1] is None


def merge_max(running: torch.Tensor, new: torch.Tensor, valid: torch.Tensor | None) -> None:
    """running = max(running, new) where ``valid`` is nonzero (device-side, no sync)."""
    _lib.launch("muzo_max_merge", running.data_ptr(), new.data_ptr(), valid.data_ptr() if valid is not None else None,
                                int(running.numel()), _lib.stream_ptr(running.device))


def to_host(tensors: list[torch.Tensor]) -> list[np.ndarray]:
    if not tensors:
        return []
    flat = torch.cat([t.reshape(-1) for t in tensors]).cpu().numpy()
    out, off = [], 0
    for t in tensors:
        out.append(flat[off: off + t.numel()].copy())
        off += t.numel()
    return out


# ---------------------------------------------------------------- scaling


def pow_factors(gamma: np.ndarray, exponent: float, dtype: torch.dtype) -> np.ndarray:
    """gamma ** exponent in fp32 (correctly rounded from float64), then rounded to ``dtype``
    the way ``.to(dtype)`` does; returned as fp32 values."""
    f = np.power(np.asarray(gamma, np.float64), float(exponent)).astype(np.float32)
    return torch.from_numpy(f).to(dtype).float().numpy()


def scale_rows(weight: torch.Tensor, groups: int, rows_per_group: int, factors: np.ndarray, mask: np.ndarray) -> None:
    """Rows of group g of ``weight`` *= factors[g] where mask[g] (qk_clip.py:289-308)."""
    scale_rows_many([(weight, groups, rows_per_group, factors, mask)])


def scale_rows_many(jobs: list) -> None:
    """Several row scalings ``(weight, groups, rows_per_group, factors, mask)``: the factors and
    masks of all jobs on a device go up in one host-to-device copy, then one launch per weight
    (a QK-Clip apply scales two matrices per attention layer: 160 for an 80-layer model)."""
    by_device: dict = {}
    for job in jobs:
        weight = job[0]
        _check_cuda(weight)
        if not weight.is_contiguous():
            raise ValueError("QK-Clip scaling expects contiguous projection weights")
        by_device.setdefault(weight.device, []).append(job)
    for dev, items in by_device.items():
        parts, offsets, off = [], [], 0
        for weight, groups, rows_per_group, factors, mask in items:
            offsets.append(off)
            parts.append(np.asarray(factors, np.float32).reshape(-1)[:groups].view(np.uint8))
            parts.append(np.asarray(mask, np.int32).reshape(-1)[:groups].view(np.uint8))
            off += 8 * int(groups)
        buf = torch.from_numpy(np.concatenate(parts)).to(dev)
        base = buf.data_ptr()
        stream = _lib.stream_ptr(dev)
        for (weight, groups, rows_per_group, _f, _m), o in zip(items, offsets):
            fptr = base + o
            _lib.launch("muzo_qk_scale_rows", weight.data_ptr(), _lib.dtype_code(weight.dtype), int(groups),
                        int(rows_per_group), int(weight.shape[1]), fptr, fptr + 4 * int(groups), stream)


# ---------------------------------------------------------------- fused attention

_ATTN_STATUS: dict[int, torch.Tensor] = {}


def attention_status(device: torch.device) -> torch.Tensor:
    """Two device int32 words per GPU: [0] the first nonzero timeout code of a fused attention
    launch, [1] the stall request (0; tests set a role's code to make its first wait expire)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ATTN_STATUS.get(idx)
    if t is None:
        t = torch.zeros(2, dtype=torch.int32, device=device)
        _ATTN_STATUS[idx] = t
    return t


def check_attention_status(device: torch.device) -> None:
    """Raise if a fused attention launch on `device` reported an expired wait (reads one word)."""
    if device.type != "cuda" or not _ATTN_STATUS:
        return
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ATTN_STATUS.get(idx)
    if t is not None and int(t[0].item()) != 0:
        code = int(t[0].item())
        t[0].zero_()
        raise _lib.MuzoError(f"fused attention reported status {code} (a bounded wait expired); the outputs of "
                             "the forward that ran it are unspecified")


def fused_attention_eligible(query, key, value, dropout: float) -> bool:
    """True when the tcgen05 attention kernel can take this call: bf16/fp16 CUDA states with head
    dim 64 or 128, D contiguous, strides of multiples of 8 elements, 16-byte aligned bases, no
    dropout and no gradient needed."""
    if dropout or query.device.type != "cuda" or query.dtype not in (torch.bfloat16, torch.float16):
        return False
    if key.dtype != query.dtype or value.dtype != query.dtype or query.shape[-1] not in (64, 128):
        return False
    if torch.is_grad_enabled() and (query.requires_grad or key.requires_grad or value.requires_grad):
        return False
    if query.shape[1] % key.shape[1] != 0 or value.shape[:3] != key.shape[:3] or value.shape[-1] != query.shape[-1]:
        return False
    for t in (query, key, value):
        if t.stride(-1) != 1 or any(int(st) % 8 for st in t.stride()[:3]) or t.data_ptr() % 16:
            return False
    return True


def attention_max(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scaling: float, causal: bool,
                  key_lo: torch.Tensor | None = None, key_hi: torch.Tensor | None = None,
                  record: bool = True) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor | None]:
    """softmax(scaling * Q K^T) V on the tensor cores for Q [B, Hq, Sq, D], K, V [B, Hkv, Sk, D]
    (transformers' transposed views), returned as [B, Sq, Hq, D] (the layout attention functions
    return); with ``record``, also the per-head max of the eager pre-softmax logits and a validity
    word, on the device. ``key_lo``/``key_hi`` (int32 per batch) bound the visible keys."""
    b, hq, sq, d = (int(v) for v in query.shape)
    hkv, sk = int(key.shape[1]), int(key.shape[2])
    dev = query.device
    out = torch.empty((b, sq, hq, d), dtype=query.dtype, device=dev)
    smax = torch.empty(hq, dtype=torch.float32, device=dev) if record else None
    valid = torch.empty(1, dtype=torch.int32, device=dev) if record else None
    status = attention_status(dev)
    _lib.launch("muzo_attention_max", query.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr(),
                _lib.dtype_code(query.dtype), b, hq, hkv, sq, sk, d,
                query.stride(0), query.stride(1), query.stride(2), key.stride(0), key.stride(1), key.stride(2),
                value.stride(0), value.stride(1), value.stride(2), sq * hq * d, d, hq * d,
                1 if causal else 0, float(scaling),
                key_lo.data_ptr() if key_lo is not None else None, key_hi.data_ptr() if key_hi is not None else None,
                smax.data_ptr() if smax is not None else None, valid.data_ptr() if valid is not None else None,
                status.data_ptr(), _lib.stream_ptr(dev))
    return out, smax, valid


# ---------------------------------------------------------------- probe attention


def _probe_attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
    """Attention function of the probe and of training-time capture: SDPA computes the output
    (and its backward); while a QK-Clip capture is active, the library's max-logit kernel reads
    the same post-RoPE query and key states and records the per-head max of the pre-softmax
    logits. With MUZO_FUSED_ATTENTION=1, a capture call that qualifies (bf16/fp16, head dim 64 or
    128, no gradient, no mask, the causal mask or a padding mask) runs one tensor-core kernel for
    the output and the maxima instead (Q K^T formed once; a query row without a visible key gets
    zeros, as SDPA returns for it). Outside a capture it is SDPA alone."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    ctrl = _ACTIVE.get()
    if scaling is None:
        scaling = query.shape[-1] ** -0.5
    if ctrl is not None and os.environ.get("MUZO_FUSED_ATTENTION", "0") == "1":
        # one kernel for the attention and the capture when the call qualifies: no mask (the
        # module's causality) or a causal / padding mask as key ranges. Off by default: on one Llama-3-70B layer
        # it takes 0.378 ms, level with SDPA plus the separate max-logit kernel (0.377 ms)
        mask = attention_mask if attention_mask is not None and attention_mask.ndim == 4 else None
        sq = query.shape[2]
        ranges = None if mask is None else mask_key_ranges(mask, query.shape[0], sq, key.shape[2])
        name = ctrl.module_name(module)
        if name is not None and (mask is None or ranges is not None) and \
                fused_attention_eligible(query, key, value, dropout):
            if ranges is None:
                causal, lo, hi = bool(getattr(module, "is_causal", True)) and sq > 1, None, None
            else:
                causal, lo, hi = ranges
            with torch.no_grad():
                out, smax, valid = attention_max(query, key, value, float(scaling), causal, lo, hi)
            ctrl.record_max(name, smax, valid)
            return out, None
    if ctrl is not None:
        with torch.no_grad():
            sq = query.shape[2]
            mask = attention_mask if attention_mask is not None and attention_mask.ndim == 4 else None
            # no mask: SDPA runs causal when the module is causal and there is more than one query
            causal = True if mask is not None else bool(getattr(module, "is_causal", True)) and sq > 1
            ctrl.record_qk(module, query.detach(), key.detach(), float(scaling), causal, mask)
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                  **kwargs)


def ensure_probe_registered() -> str:
    """Register the probe attention (with the eager mask format) with transformers once."""
    global _REGISTERED
    from .qk_clip import PROBE_ATTENTION

    if not _REGISTERED:
        from transformers import AttentionInterface
        from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, eager_mask

        AttentionInterface.register(PROBE_ATTENTION, _probe_attention)
        ALL_MASK_ATTENTION_FUNCTIONS.register(PROBE_ATTENTION, eager_mask)
        _REGISTERED = True
    return PROBE_ATTENTION


_TRAINING_REGISTERED = False


def ensure_training_registered() -> str:
    """Register the training-time capture attention with SDPA's mask format (no mask for plain
    causal attention, so SDPA keeps its fused causal kernels) once."""
    global _TRAINING_REGISTERED
    from .qk_clip import CAPTURE_ATTENTION

    if not _TRAINING_REGISTERED:
        from transformers import AttentionInterface
        from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, sdpa_mask

        AttentionInterface.register(CAPTURE_ATTENTION, _probe_attention)
        ALL_MASK_ATTENTION_FUNCTIONS.register(CAPTURE_ATTENTION, sdpa_mask)
        _TRAINING_REGISTERED = True
    return CAPTURE_ATTENTION
