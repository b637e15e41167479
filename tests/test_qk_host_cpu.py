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
    real = _qk._key_ranges_uncached
    monkeypatch.setattr(_qk, "_key_ranges_uncached", lambda *a: calls.append(1) or real(*a))
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


def _padding_keep(lens_lo, lens_hi, sq, sk, causal):
    """[B, 1, Sq, Sk] boolean mask: batch row b attends to keys [lo_b, hi_b) (and causally)."""
    j = torch.arange(sk)
    rows = []
    for lo, hi in zip(lens_lo, lens_hi):
        r = ((j >= lo) & (j < hi))[None, :].expand(sq, sk)
        if causal:
            r = r & _causal_keep(sq, sk)
        rows.append(r)
    return torch.stack(rows)[:, None]


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("form", ["bool", "additive_f32", "additive_bf16", "additive_f16"])
def test_padding_masks_become_key_ranges(causal, form):
    from muzo_clip_b200._qk import mask_key_ranges

    sq = sk = 12
    lo, hi = [0, 3, 0, 5], [12, 12, 9, 10]      # none, left, right, both
    keep = _padding_keep(lo, hi, sq, sk, causal)
    if form == "bool":
        mask = keep
    else:
        dt = {"additive_f32": torch.float32, "additive_bf16": torch.bfloat16, "additive_f16": torch.float16}[
            form]
        mask = torch.zeros(keep.shape, dtype=dt).masked_fill(~keep, torch.finfo(dt).min)
    r = mask_key_ranges(mask, 4, sq, sk)
    assert r is not None
    got_causal, got_lo, got_hi = r
    assert got_causal == causal
    assert got_lo.tolist() == lo and got_hi.tolist() == hi
    assert got_lo.dtype == torch.int32 and got_lo.is_contiguous()


def test_padding_mask_rows_without_keys_and_unmasked_rows():
    """Left padding in a causal model: the padding queries see no key. transformers may let such
    rows attend everywhere in SDPA's boolean form; both forms give the same ranges."""
    from muzo_clip_b200._qk import mask_key_ranges

    sq = sk = 8
    keep = _padding_keep([0, 3], [8, 8], sq, sk, True)
    unmasked = keep.clone()
    unmasked[1, :, :3, :] = True
    for m in (keep, unmasked):
        causal, lo, hi = mask_key_ranges(m, 2, sq, sk)
        assert causal and lo.tolist() == [0, 3] and hi.tolist() == [8, 8]


def test_other_masks_are_not_key_ranges():
    from muzo_clip_b200._qk import mask_key_ranges

    sq = sk = 8
    keep = _padding_keep([0, 0], [8, 8], sq, sk, True)
    holes = keep.clone()
    holes[0, :, :, 2] = False                    # a masked key inside the visible range
    assert mask_key_ranges(holes, 2, sq, sk) is None
    blocks = keep.clone()
    blocks[:, :, 4:, :4] = False                 # block-diagonal (packed sequences)
    assert mask_key_ranges(blocks, 2, sq, sk) is None
    per_head = keep.expand(2, 3, sq, sk)         # a mask per head
    assert mask_key_ranges(per_head, 2, sq, sk) is None
    bias = torch.zeros(2, 1, sq, sk).masked_fill(~keep, -1e30)
    bias[0, 0, 5, 1] = -0.5                      # a bias, not a mask
    assert mask_key_ranges(bias, 2, sq, sk) is None
    # one mask row for the whole batch expands to every batch row
    causal, lo, hi = mask_key_ranges(_padding_keep([2], [7], sq, sk, False), 3, sq, sk)
    assert not causal and lo.tolist() == [2, 2, 2] and hi.tolist() == [7, 7, 7]
    # the plain causal mask: no ranges
    assert mask_key_ranges(keep, 2, sq, sk) == (True, None, None)


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

    monkeypatch.setattr(qk, "scale_rows_many", lambda jobs: [_cpu_scale_rows(*job) for job in jobs])
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
