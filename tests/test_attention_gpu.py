"""The tensor-core attention forward with the per-head max-logit side output (muzo_attention_max).

Output: against softmax(scale * Q K^T) V computed in fp32 from the same bf16/fp16 inputs, within
a bound tied to SDPA's own error on the same inputs (both keep P in the input dtype). Side
output: against the eager pre-softmax logits of qk_clip.py:173-196 (the reference's capture),
within one ulp of the dtype per head. Causal (end-aligned), GQA, Sq != Sk, per-batch key ranges
(padding), rows without a visible key (zeros), head dims 64 and 128.
"""

from __future__ import annotations

import math

import pytest
import torch

import torch_reference as tr

pytestmark = pytest.mark.gpu


def _reference(q, k, v, scale, causal, lo=None, hi=None):
    """fp32 attention over the visible keys, [B, Sq, Hq, D]; rows with no visible key are 0.
    Also the boolean visibility mask [B, 1, Sq, Sk]."""
    b, hq, sq, d = q.shape
    hkv, sk = k.shape[1], k.shape[2]
    group = hq // hkv
    kf = k.float().repeat_interleave(group, dim=1)
    vf = v.float().repeat_interleave(group, dim=1)
    logits = torch.matmul(q.float(), kf.transpose(2, 3)) * scale
    i = torch.arange(sq, device=q.device)[:, None] + (sk - sq)
    j = torch.arange(sk, device=q.device)[None, :]
    vis = torch.ones((b, 1, sq, sk), dtype=torch.bool, device=q.device)
    if causal:
        vis = vis & (j <= i)
    if lo is not None:
        for bi in range(b):
            vis[bi] &= (j >= int(lo[bi])) & (j < int(hi[bi]))
    logits = logits.masked_fill(~vis, float("-inf"))
    p = torch.softmax(logits, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    out = torch.matmul(p, vf)
    return out.transpose(1, 2).contiguous(), vis


def _visible_max(q, k, scale, vis, dtype):
    """Per-head max of the eager logits round(round(q . k) * scale) over the visible keys."""
    group = q.shape[1] // k.shape[1]
    kr = k.repeat_interleave(group, dim=1)
    logits = (torch.matmul(q, kr.transpose(2, 3)) * scale).float()  # eager: matmul in dtype, times scale
    logits = logits.masked_fill(~vis, float("-inf"))
    return logits.amax(dim=(0, 2, 3)).cpu()


CASES = [  # b, hq, hkv, sq, sk, d, causal
    (2, 8, 2, 300, 300, 64, True),
    (1, 4, 4, 1000, 1000, 128, True),
    (2, 6, 3, 257, 257, 128, False),
    (1, 4, 2, 100, 356, 128, True),     # Sq < Sk: end-aligned causal window
    (3, 2, 1, 130, 130, 64, False),
    (1, 2, 2, 128, 64, 64, True),      # Sq > Sk: the first rows see no key
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,hq,hkv,sq,sk,d,causal", CASES)
def test_fused_attention_output_and_max(device, dtype, b, hq, hkv, sq, sk, d, causal):
    from muzo_clip_b200 import _qk

    g = torch.Generator(device="cpu").manual_seed(b * 1000 + hq * 10 + sq + d)
    # transformers' layout: [B, S, H, D] viewed as [B, H, S, D]
    q = (torch.randn((b, sq, hq, d), generator=g) * 1.5).to(dtype).to(device).transpose(1, 2)
    k = (torch.randn((b, sk, hkv, d), generator=g) * 1.5).to(dtype).to(device).transpose(1, 2)
    v = torch.randn((b, sk, hkv, d), generator=g).to(dtype).to(device).transpose(1, 2)
    scale = d ** -0.5
    out, smax, valid = _qk.attention_max(q, k, v, scale, causal)
    torch.cuda.synchronize()
    ref, vis = _reference(q, k, v, scale, causal)
    # SDPA's own error on the same inputs (explicit visibility mask; rows without a visible key
    # excluded: SDPA returns NaN there)
    group = hq // hkv
    sd = torch.nn.functional.scaled_dot_product_attention(
        q, k.repeat_interleave(group, dim=1), v.repeat_interleave(group, dim=1), attn_mask=vis, scale=scale)
    sd = sd.transpose(1, 2).float()
    rows = vis[:, 0].any(dim=-1)[:, :, None, None]              # [B, Sq, 1, 1]
    err = (out.float() - ref).abs()
    sd_err = torch.nan_to_num((sd - ref).abs(), nan=0.0) * rows
    assert float(err.max()) <= 2.0 * float(sd_err.max()) + 2e-3, (float(err.max()), float(sd_err.max()))
    assert torch.equal(out[~rows.expand_as(out)], torch.zeros_like(out[~rows.expand_as(out)]))
    assert int(valid.item()) == 1
    want = _visible_max(q, k, scale, vis, dtype)
    want = want.to(dtype).float()
    bits = 7 if dtype == torch.bfloat16 else 10
    got = smax.cpu()
    fin = torch.isfinite(want)
    ulp = torch.pow(2.0, torch.floor(torch.log2(want[fin].abs().clamp_min(2.0 ** -126))) - bits)
    assert bool(((got[fin] - want[fin]).abs() <= ulp).all()), (got, want)
    assert bool((got[~fin] == float("-inf")).all())


@pytest.mark.parametrize("causal", [True, False])
def test_fused_attention_key_ranges(device, causal):
    """Per-batch visible key ranges [lo, hi) (left and right padding): output and maxima over the
    visible keys only."""
    from muzo_clip_b200 import _qk

    dtype = torch.bfloat16
    b, hq, hkv, s, d = 3, 4, 2, 300, 128
    g = torch.Generator(device="cpu").manual_seed(31)
    q = torch.randn((b, s, hq, d), generator=g).to(dtype).to(device).transpose(1, 2)
    k = torch.randn((b, s, hkv, d), generator=g).to(dtype).to(device).transpose(1, 2)
    v = torch.randn((b, s, hkv, d), generator=g).to(dtype).to(device).transpose(1, 2)
    lo = torch.tensor([0, 37, 150], dtype=torch.int32, device=device)
    hi = torch.tensor([300, 300, 290], dtype=torch.int32, device=device)
    scale = d ** -0.5
    out, smax, valid = _qk.attention_max(q, k, v, scale, causal, lo, hi)
    torch.cuda.synchronize()
    ref, vis = _reference(q, k, v, scale, causal, lo.cpu(), hi.cpu())
    rows = vis[:, 0].any(dim=-1)[:, :, None, None]
    err = ((out.float() - ref).abs() * rows).max()
    assert float(err) <= 2e-2, float(err)
    assert torch.equal(out[~rows.expand_as(out)], torch.zeros_like(out[~rows.expand_as(out)]))
    want = _visible_max(q, k, scale, vis, dtype).to(dtype).float()
    ulp = torch.pow(2.0, torch.floor(torch.log2(want.abs().clamp_min(2.0 ** -126))) - 7)
    assert bool(((smax.cpu() - want).abs() <= ulp).all()) and int(valid.item()) == 1


def test_fused_attention_llama3_70b_layer(device):
    """One Llama-3-70B-shaped attention layer (B = 1, S = 4096, 64 query / 8 KV heads of 128,
    causal, bf16): output against SDPA, maxima against the eager logits."""
    from muzo_clip_b200 import _qk

    g = torch.Generator(device=device).manual_seed(70)
    q = torch.randn((1, 4096, 64, 128), generator=g, device=device).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn((1, 4096, 8, 128), generator=g, device=device).to(torch.bfloat16).transpose(1, 2)
    v = torch.randn((1, 4096, 8, 128), generator=g, device=device).to(torch.bfloat16).transpose(1, 2)
    scale = 128 ** -0.5
    out, smax, valid = _qk.attention_max(q, k, v, scale, True)
    sd = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale, enable_gqa=True)
    sd = sd.transpose(1, 2)
    torch.cuda.synchronize()
    err = (out.float() - sd.float()).abs()
    assert float(err.max()) <= 3e-2 and float(err.mean()) <= 2e-3, (float(err.max()), float(err.mean()))
    want = tr.qk_head_max(tr.eager_logits(q, k, scale, True))
    ulp = torch.pow(2.0, torch.floor(torch.log2(want.abs().clamp_min(2.0 ** -126))) - 7)
    assert bool(((smax.cpu() - want).abs() <= ulp).all()) and int(valid.item()) == 1
    assert math.isfinite(float(smax.max()))


def test_fused_attention_flags_nonfinite_logits(device):
    from muzo_clip_b200 import _qk

    q = torch.randn((1, 2, 200, 64), device=device, dtype=torch.bfloat16)
    k = torch.randn((1, 2, 200, 64), device=device, dtype=torch.bfloat16)
    v = torch.randn((1, 2, 200, 64), device=device, dtype=torch.bfloat16)
    q[0, 1, 3, 5] = float("inf")
    _, _, valid = _qk.attention_max(q, k, v, 0.125, True)
    assert int(valid.item()) == 0


@pytest.mark.parametrize("role", [1, 2, 3])
def test_fused_attention_bounded_waits_expire(device, role):
    """A stall request (status word 1) makes one role's first wait expire: the producer (1), the
    MMA issuer (2) or the softmax warps (3). The kernel records that role's code, drains its loads
    and MMAs, frees TMEM and returns; the Python check raises; the next launch on the same context
    computes the right result."""
    from muzo_clip_b200 import _lib, _qk

    g = torch.Generator(device="cpu").manual_seed(5)
    q = torch.randn((1, 300, 2, 64), generator=g).to(torch.bfloat16).to(device).transpose(1, 2)
    k = torch.randn((1, 300, 2, 64), generator=g).to(torch.bfloat16).to(device).transpose(1, 2)
    v = torch.randn((1, 300, 2, 64), generator=g).to(torch.bfloat16).to(device).transpose(1, 2)
    status = _qk.attention_status(device)
    status.zero_()
    status[1] = role
    try:
        _qk.attention_max(q, k, v, 0.125, True)
        torch.cuda.synchronize()
        assert int(status[0].item()) == role
        with pytest.raises(_lib.MuzoError):
            _qk.check_attention_status(device)
        assert int(status[0].item()) == 0
    finally:
        status[1] = 0
    out, smax, valid = _qk.attention_max(q, k, v, 0.125, True)
    torch.cuda.synchronize()
    _qk.check_attention_status(device)
    ref, vis = _reference(q, k, v, 0.125, True)
    assert float((out.float() - ref).abs().max()) <= 3e-2
    assert int(valid.item()) == 1
