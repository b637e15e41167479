"""Host-side pieces of the QK-Clip capture that need no GPU: mask classification and the
conversion of SDPA's boolean masks to eager attention's additive form."""

from __future__ import annotations

import pytest
import torch


def _causal_keep(sq, sk):
    i = torch.arange(sq)[:, None] + (sk - sq)
    return torch.arange(sk)[None, :] <= i


def test_plain_causal_detection_additive_and_boolean():
    from muzo_clip_b200._qk import _is_plain_causal

    keep = _causal_keep(6, 9)[None, None]
    additive = torch.zeros((1, 1, 6, 9)).masked_fill(~keep, torch.finfo(torch.bfloat16).min)
    assert _is_plain_causal(additive, 6, 9)
    assert _is_plain_causal(keep, 6, 9)
    padded = keep.clone()
    padded[..., 0] = False            # a padding key
    assert not _is_plain_causal(padded, 6, 9)
    assert not _is_plain_causal(additive[..., :8], 6, 9)   # shape mismatch


def test_plain_causal_test_is_cached_per_mask_and_version(monkeypatch):
    from muzo_clip_b200 import _qk

    calls = []
    real = _qk._plain_causal_uncached
    monkeypatch.setattr(_qk, "_plain_causal_uncached", lambda *a: calls.append(1) or real(*a))
    i = torch.arange(5)[:, None]
    mask = torch.zeros(1, 1, 5, 5).masked_fill(torch.arange(5)[None, :] > i, torch.finfo(torch.float32).min)
    for _ in range(4):  # one mask, every layer of a forward
        assert _qk._is_plain_causal(mask, 5, 5)
    assert len(calls) == 1
    assert not _qk._is_plain_causal(mask, 5, 6) and len(calls) == 2   # other shape: computed
    mask[0, 0, 4, 0] = torch.finfo(torch.float32).min                  # in place: new version
    assert not _qk._is_plain_causal(mask, 5, 5) and len(calls) == 3
    other = mask.clone()                                                # another tensor
    assert not _qk._is_plain_causal(other, 5, 5) and len(calls) == 4
    with torch.inference_mode():                                        # no version counter
        inf_mask = torch.zeros(1, 1, 2, 2)
    assert not _qk._is_plain_causal(inf_mask, 2, 2)


def test_boolean_mask_to_eager_form_remasks_unmasked_padding_rows():
    from muzo_clip_b200._qk import eager_additive_mask

    sq = sk = 5
    keep = _causal_keep(sq, sk).clone()[None, None].repeat(2, 1, 1, 1)
    keep[1, :, :, :2] = False          # left padding of two tokens in batch row 1
    # transformers' SDPA fix: the fully masked padding query rows attend everywhere
    fixed = keep.clone()
    fixed[1, :, :2, :] = True
    add = eager_additive_mask(fixed, causal=True, dtype=torch.float32)
    mn = torch.finfo(torch.float32).min
    assert torch.equal(add == 0, keep)  # exactly eager's visibility again
    assert bool((add[~keep] == mn).all())
    # non-causal masks are converted as they are
    add_nc = eager_additive_mask(fixed, causal=False, dtype=torch.bfloat16)
    assert torch.equal(add_nc == 0, fixed)


def test_capture_attention_needs_a_transformers_model():
    pytest.importorskip("transformers")
    from muzo_clip_b200 import use_qk_capture_attention

    with pytest.raises(ValueError):
        use_qk_capture_attention(torch.nn.Linear(4, 4))


def _attn_model(hidden, hq, hkv, hd, dtype):
    torch.manual_seed(3)
    model = torch.nn.Module()
    model.layers = torch.nn.ModuleList()
    for _ in range(2):
        blk = torch.nn.Module()
        blk.self_attn = torch.nn.Module()
        blk.self_attn.q_proj = torch.nn.Linear(hidden, hq * hd, bias=False)
        blk.self_attn.k_proj = torch.nn.Linear(hidden, hkv * hd, bias=False)
        model.layers.append(blk)
    return model.to(dtype)


def _cpu_scale_rows(weight, groups, rows_per_group, factors, mask):
    """The row-scaling kernel's arithmetic on the CPU: fp32 product rounded to the weight dtype."""
    w = weight.view(groups, rows_per_group, -1)
    for g in range(groups):
        if mask[g]:
            w[g] = (w[g].float() * float(factors[g])).to(weight.dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("hq,hkv,q_rows", [(4, 2, None), (4, 4, None), (4, 2, 4 * 8 + 8)])
def test_qk_scaling_host_logic_matches_reference(monkeypatch, dtype, hq, hkv, q_rows):
    """Which heads and KV groups are scaled, by which rounded factors, and the returned
    statistics (qk_clip.py:198-322) — the reference on CPU tensors against this controller with
    its device row-scaling replaced by the same arithmetic on the CPU. q_rows not divisible by
    the head count exercises the whole-matrix fallback."""
    import copy
    import sys

    from reference_pkg import reference_path

    ref_root = reference_path()
    if ref_root is None:
        pytest.skip("reference package not available (MUZO_REFERENCE_PATH / baseline/_ref)")
    sys.path.insert(0, str(ref_root))
    from muzo_clip.qk_clip import QKClipController as RefController

    import muzo_clip_b200._qk as qk
    from muzo_clip_b200.qk_clip import QKClipController

    monkeypatch.setattr(qk, "scale_rows", _cpu_scale_rows)
    hd = 8
    mine_model = _attn_model(32, hq, hkv, hd, dtype)
    if q_rows is not None:  # a q projection whose rows do not split into the heads
        for blk in mine_model.layers:
            blk.self_attn.q_proj = torch.nn.Linear(32, q_rows, bias=False).to(dtype)
    ref_model = copy.deepcopy(mine_model)
    tau, alpha = 10.0, 0.5
    ref, mine = RefController(ref_model, tau=tau, alpha=alpha), QKClipController(mine_model, tau=tau, alpha=alpha)
    smax = {"layers.0.self_attn": torch.tensor([3.0, 25.0, 9.5, 60.0][:hq]),
            "layers.1.self_attn": torch.tensor([1.0, 2.0, 3.0, 4.0][:hq])}
    ref._captured_smax = {k: v.clone() for k, v in smax.items()}
    mine._captured_smax = {k: v.clone() for k, v in smax.items()}
    a, b = ref.apply(), mine.apply()
    assert (a.enabled, a.exact_logits, a.fallback_used, a.qk_clip_count) == \
        (b.enabled, b.exact_logits, b.fallback_used, b.qk_clip_count)
    assert abs(a.qk_smax_max - b.qk_smax_max) <= 1e-6 * a.qk_smax_max
    for (n1, p1), (n2, p2) in zip(ref_model.named_parameters(), mine_model.named_parameters()):
        assert n1 == n2
        diff = (p1.float() - p2.float()).abs()
        ulp = p1.float().abs().clamp_min(1e-30) * (2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -22)
        assert bool((diff <= ulp).all()), n1   # the factors agree to one rounding of gamma ** alpha
