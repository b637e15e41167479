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
