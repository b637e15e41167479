"""QK-Clip on the GPU against the reference's eager-attention capture (qk_clip.py:161-322)."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

import torch_reference as tr

pytestmark = pytest.mark.gpu


def _ulp(x: torch.Tensor, bits: int) -> torch.Tensor:
    ax = x.abs().clamp_min(2.0 ** -126)
    return torch.pow(2.0, torch.floor(torch.log2(ax)) - bits)


@pytest.fixture(params=["pair", "single"])
def qk_kernel(request, monkeypatch):
    """bf16 / fp16 run on the CTA-pair kernel (256 x 256 tiles, query block resident) unless
    MUZO_QK_PAIR=0 selects the one-SM kernel: both are checked."""
    monkeypatch.setenv("MUZO_QK_PAIR", "1" if request.param == "pair" else "0")
    return request.param


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("b,hq,hkv,sq,sk,d", [(2, 8, 2, 100, 100, 64), (1, 4, 4, 64, 64, 128), (2, 6, 1, 33, 70, 32),
                                             (1, 8, 2, 1000, 1000, 128), (1, 2, 1, 300, 700, 96),
                                             (1, 4, 1, 520, 520, 256), (3, 2, 2, 257, 257, 64)])
def test_qk_max_matches_eager_logits(device, qk_kernel, dtype, causal, b, hq, hkv, sq, sk, d):
    from muzo_clip_b200 import _qk

    g = torch.Generator(device="cpu").manual_seed(b * 100 + hq + sq)
    # HF layout: [B, S, H, D] viewed as [B, H, S, D] (non-contiguous, D contiguous)
    q = (torch.randn((b, sq, hq, d), generator=g) * 2).to(dtype).to(device).transpose(1, 2)
    k = (torch.randn((b, sk, hkv, d), generator=g) * 2).to(dtype).to(device).transpose(1, 2)
    scale = d ** -0.5
    ref = tr.qk_head_max(tr.eager_logits(q, k, scale, causal and sq <= sk))
    got, valid = _qk.qk_head_max(q, k, scale, causal and sq <= sk, None)
    torch.cuda.synchronize()
    assert int(valid.item()) == 1
    got = got.cpu()
    bits = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 19}[dtype]
    assert bool(((got - ref).abs() <= _ulp(ref, bits)).all()), (got, ref)


def _padded_keep(lo, hi, sq, sk, causal, device):
    j = torch.arange(sk, device=device)
    rows = []
    for a, b in zip(lo, hi):
        r = ((j >= a) & (j < b))[None, :].expand(sq, sk)
        if causal:
            r = r & (j[None, :] <= torch.arange(sq, device=device)[:, None] + (sk - sq))
        rows.append(r)
    return torch.stack(rows)[:, None]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("form", ["bool", "additive"])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("b,hq,hkv,sq,sk,d,lo,hi", [
    (3, 8, 2, 300, 300, 64, [0, 37, 0], [300, 300, 211]),         # none, left, right padding
    (2, 4, 4, 1000, 1000, 128, [500, 0], [1000, 129]),             # long left / right padding
    (2, 2, 1, 200, 460, 96, [259, 3], [460, 300]),                 # Sq < Sk, both sides
    (2, 4, 1, 520, 520, 256, [0, 130], [520, 520]),                # head dim 256
])
def test_qk_max_with_padding_masks(device, qk_kernel, monkeypatch, dtype, form, causal, b, hq, hkv, sq, sk, d, lo,
                                   hi):
    """Padding masks (per batch row a range of visible keys, causal or not, in SDPA's boolean or
    eager's additive form) run on the same kernels with per-batch key ranges: maxima equal the
    eager capture's amax of logits + mask (qk_clip.py:186-196), without the S x S logits."""
    from muzo_clip_b200 import _qk

    g = torch.Generator(device="cpu").manual_seed(b * 7 + sq + d)
    q = (torch.randn((b, sq, hq, d), generator=g) * 2).to(dtype).to(device).transpose(1, 2)
    k = (torch.randn((b, sk, hkv, d), generator=g) * 2).to(dtype).to(device).transpose(1, 2)
    scale = d ** -0.5
    keep = _padded_keep(lo, hi, sq, sk, causal, device)
    additive = torch.zeros(keep.shape, dtype=dtype, device=device).masked_fill(~keep, torch.finfo(dtype).min)
    mask = keep if form == "bool" else additive

    def no_logits(*a, **kw):
        raise AssertionError("a padding mask must not materialise the logits")

    monkeypatch.setattr(_qk, "logits_head_max", no_logits)
    got, valid = _qk.qk_head_max(q, k, scale, True, mask)
    torch.cuda.synchronize()
    assert int(valid.item()) == 1
    kr = k.repeat_interleave(hq // hkv, dim=1)
    want = ((torch.matmul(q, kr.transpose(2, 3)) * scale) + additive).float().amax(dim=(0, 2, 3)).cpu()
    bits = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 19}[dtype]
    assert bool(((got.cpu() - want).abs() <= _ulp(want, bits)).all()), (got, want)


@pytest.mark.parametrize("bad", [float("inf"), float("-inf"), float("nan")])
def test_qk_max_flags_nonfinite(device, qk_kernel, bad):
    from muzo_clip_b200 import _qk

    q = torch.randn((1, 2, 300, 64), device=device, dtype=torch.bfloat16)
    k = torch.randn((1, 2, 300, 64), device=device, dtype=torch.bfloat16)
    q[0, 1, 3, 5] = bad
    _, valid = _qk.qk_head_max(q, k, 0.2, True, None)
    assert int(valid.item()) == 0
    q[0, 1, 3, 5] = 0.0
    _, valid = _qk.qk_head_max(q, k, 0.2, True, None)
    assert int(valid.item()) == 1


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_logits_head_max_and_guarded_merge(device, dtype):
    from muzo_clip_b200 import _qk

    logits = (torch.randn((2, 5, 17, 23), device=device) * 4).to(dtype)
    got, valid = _qk.logits_head_max(logits)
    assert torch.equal(got.cpu(), tr.qk_head_max(logits)) and int(valid.item()) == 1
    running = torch.full((5,), -1.0e9, device=device)
    _qk.merge_max(running, got, valid)
    assert torch.equal(running.cpu(), got.cpu())
    bad = logits.clone()
    bad[1, 2, 3, 4] = float("nan")
    g2, v2 = _qk.logits_head_max(bad)
    before = running.clone()
    _qk.merge_max(running, g2 + 100.0, v2)  # dropped: the capture had a non-finite logit
    assert int(v2.item()) == 0 and torch.equal(running, before)


def _tiny_llama(dtype, device, kv_heads=2):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=kv_heads,
                      intermediate_size=688, vocab_size=1024, attn_implementation="sdpa", initializer_range=0.02)
    return LlamaForCausalLM(cfg).to(dtype=dtype, device=device).eval()


def _reference_capture(model, ids):
    """The reference's capture (qk_clip.py:91-118, 173-196) restated: eager attention, softmax
    input of each attention module reduced to per-head maxima."""
    import torch.nn.functional as F

    names = {id(m): n for n, m in model.named_modules() if hasattr(m, "q_proj") and hasattr(m, "k_proj")}
    stack, captured = [], {}
    hooks = []
    for mod_id, name in names.items():
        mod = next(m for m in model.modules() if id(m) == mod_id)
        hooks.append(mod.register_forward_pre_hook(lambda m, a, name=name: stack.append(name)))
        hooks.append(mod.register_forward_hook(lambda m, a, o: stack.pop() and None))  # must return None
    orig = F.softmax

    def patched(inp, *args, **kwargs):
        if stack and inp.ndim == 4:
            per = inp.detach().float().amax(dim=(0, 2, 3)).cpu()
            prev = captured.get(stack[-1])
            captured[stack[-1]] = per if prev is None else torch.maximum(prev, per)
        return orig(inp, *args, **kwargs)

    saved = model.config._attn_implementation
    model.config._attn_implementation = "eager"
    F.softmax = patched
    try:
        with torch.no_grad():
            model(input_ids=ids)
    finally:
        F.softmax = orig
        model.config._attn_implementation = saved
        for h in hooks:
            h.remove()
    return captured


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_probe_and_apply_matches_reference(device, dtype):
    from muzo_clip_b200 import MuZOClipOptimizer

    model = _tiny_llama(dtype, device)
    # make some heads exceed tau so clipping happens
    with torch.no_grad():
        model.model.layers[0].self_attn.q_proj.weight.mul_(40.0)
        model.model.layers[1].self_attn.k_proj.weight[:64].mul_(30.0)
    twin = copy.deepcopy(model)
    ids = torch.randint(0, 1024, (4, 64), generator=torch.Generator().manual_seed(1)).to(device)
    ref_smax = _reference_capture(twin, ids)
    tau, alpha = 5.0, 0.5
    opt = MuZOClipOptimizer(model, enable_qk_clip=True, qk_clip_tau=tau, qk_clip_alpha=alpha)
    # capture only, to compare the maxima before any scaling
    ctrl = opt.qk_clip
    ctrl.clear()
    with ctrl.force_eager_attention(True):
        with ctrl.capture():
            with torch.no_grad():
                model(input_ids=ids)
    # bf16: one ulp (rounding of the same dot product); fp32: a few ulps of accumulation order
    bits = 7 if dtype == torch.bfloat16 else 19
    assert set(ctrl._captured_smax) == set(ref_smax)
    for name, ref in ref_smax.items():
        got = ctrl._captured_smax[name].cpu()
        assert bool(((got - ref).abs() <= _ulp(ref, bits)).all()), (name, got, ref)
    stats = ctrl.apply()
    # the reference's scaling on the twin with the reference maxima
    count = 0
    smax_max = 0.0
    for name, smax in ref_smax.items():
        mod = twin.get_submodule(name)
        smax_max = max(smax_max, float(smax.max()))
        c, _ = tr.qk_scale(mod.q_proj.weight.data, mod.k_proj.weight.data, smax, tau, alpha)
        count += c
    assert stats.enabled and stats.exact_logits and not stats.fallback_used
    assert stats.qk_clip_count == count and count > 0
    assert abs(stats.qk_smax_max - smax_max) <= 2.0 ** -bits * smax_max
    for (n1, p1), (_, p2) in zip(model.named_parameters(), twin.named_parameters()):
        if "q_proj" in n1 or "k_proj" in n1:
            diff = (p1.float() - p2.float()).abs()
            assert bool((diff <= _ulp(p2.float(), bits)).all()), n1
            if dtype == torch.bfloat16:  # factors rounded to bf16 coincide almost always
                assert (p1 == p2).float().mean().item() > 0.99
        else:
            assert torch.equal(p1, p2), n1


def test_probe_reports_disabled_without_modules(device):
    from muzo_clip_b200 import MuZOClipOptimizer

    model = torch.nn.Sequential(torch.nn.Linear(8, 8)).to(device)
    opt = MuZOClipOptimizer(model, enable_qk_clip=True)
    st = opt.probe_and_apply_qk_clip(lambda: torch.tensor(1.0))
    assert st["enabled"] is False and st["disabled_reason"] == "no q_proj/k_proj attention modules found"


@pytest.mark.parametrize("fused", ["0", "1"])
@pytest.mark.parametrize("padded", [False, True])
def test_training_capture_attention(device, monkeypatch, padded, fused):
    """use_qk_capture_attention: outputs and gradients are SDPA's; the clean forward of
    estimate_projection (qk_capture_clean_forward=True) records the eager maxima exactly, with
    and without a padding mask; apply_qk_clip_if_available then clips."""
    from muzo_clip_b200 import MuZOClipOptimizer, use_qk_capture_attention

    monkeypatch.setenv("MUZO_FUSED_ATTENTION", fused)   # SDPA + max kernel, or the fused attention kernel
    model = _tiny_llama(torch.bfloat16, device)
    with torch.no_grad():
        model.model.layers[0].self_attn.q_proj.weight.mul_(40.0)
    sdpa = copy.deepcopy(model)
    ids = torch.randint(0, 1024, (3, 48), generator=torch.Generator().manual_seed(2)).to(device)
    mask = torch.ones_like(ids)
    if padded:
        mask[1, :7] = 0  # left padding of one row
    assert use_qk_capture_attention(model) == "muzo_qk_sdpa"

    # no capture active: the same function as SDPA, forward and backward
    model.train(), sdpa.train()
    out = model(input_ids=ids, attention_mask=mask, labels=ids)
    ref = sdpa(input_ids=ids, attention_mask=mask, labels=ids)
    assert torch.equal(out.logits, ref.logits)
    out.loss.backward()
    ref.loss.backward()
    g1 = model.model.layers[0].self_attn.q_proj.weight.grad
    g2 = sdpa.model.layers[0].self_attn.q_proj.weight.grad
    assert g1 is not None and torch.equal(g1, g2)
    model.zero_grad(set_to_none=True)
    model.eval()

    twin = copy.deepcopy(sdpa)
    opt = MuZOClipOptimizer(model, enable_qk_clip=True, qk_capture_clean_forward=True, qk_clip_tau=5.0,
                            restore_exact=True, seed=3)

    def closure():
        with torch.no_grad():
            return model(input_ids=ids, attention_mask=mask, labels=ids).loss

    proj = opt.estimate_projection(closure)
    assert not proj["skipped"]
    captured = {k: v.cpu() for k, v in opt.qk_clip._captured_smax.items()}
    # reference: eager softmax inputs of the same (restored, clean) weights
    names = {id(m): n for n, m in twin.named_modules() if hasattr(m, "q_proj") and hasattr(m, "k_proj")}
    stack, want, hooks = [], {}, []
    for mod_id, name in names.items():
        mod = next(m for m in twin.modules() if id(m) == mod_id)
        hooks.append(mod.register_forward_pre_hook(lambda m, a, name=name: stack.append(name)))
        hooks.append(mod.register_forward_hook(lambda m, a, o: stack.pop() and None))
    import torch.nn.functional as F
    orig = F.softmax

    def patched(inp, *args, **kwargs):
        if stack and inp.ndim == 4:
            per = inp.detach().float().amax(dim=(0, 2, 3)).cpu()
            prev = want.get(stack[-1])
            want[stack[-1]] = per if prev is None else torch.maximum(prev, per)
        return orig(inp, *args, **kwargs)

    twin.config._attn_implementation = "eager"
    F.softmax = patched
    try:
        with torch.no_grad():
            twin(input_ids=ids, attention_mask=mask)
    finally:
        F.softmax = orig
        for h in hooks:
            h.remove()
    assert set(captured) == set(want)
    for name, ref_max in want.items():
        assert bool(((captured[name] - ref_max).abs() <= _ulp(ref_max, 7)).all()), (name, captured[name], ref_max)
    stats = opt.qk_clip.apply()  # the clip that apply_qk_clip_if_available runs after an updating step
    assert stats.enabled and stats.exact_logits and stats.qk_clip_count > 0
