"""End to end on a tiny Llama-style decoder: 2 layers, hidden 256, 4 heads, MLP 688, vocab
1024, fp32, batch 4 x seq 64 token ids, the optimizer's default hyperparameters,
normal noise, 20 SPSA steps and one QK-Clip probe — the sanity checks of the reference project's
README.md:253-258, plus every update within 2e-2 of the exact-accumulation iteration's and no
further from the reference path than the reference path is from that iteration, + 2e-2."""

from __future__ import annotations

import copy
import math

import pytest
import torch

import torch_reference as tr

pytestmark = pytest.mark.gpu


def _model(device, attn="eager"):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(1234)
    cfg = LlamaConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=4,
                      intermediate_size=688, vocab_size=1024, attn_implementation=attn, initializer_range=0.02)
    return LlamaForCausalLM(cfg).float().to(device)


def test_tiny_llama_twenty_steps_and_probe(device):
    from muzo_clip_b200 import MuZOClipOptimizer

    model = _model(device)
    ids = torch.randint(0, 1024, (4, 64), generator=torch.Generator().manual_seed(0)).to(device)
    opt = MuZOClipOptimizer(model, enable_qk_clip=True, seed=1234)
    assert len(opt.selected_parameter_names()) == 14

    def closure():
        return model(input_ids=ids, labels=ids).loss

    from exact_step import block_update_from_ns, capture_ns_outputs, exact_block_update, rel

    projections, steps = [], []
    twin = copy.deepcopy(model)
    named_twin = [(n, p) for n, p in twin.named_parameters() if n in set(opt.selected_parameter_names())]
    params = dict(model.named_parameters())
    max_u = max_stored = 0.0
    for _ in range(20):
        proj = opt.estimate_projection(closure)
        projections.append(proj)
        # the reference path's perturb / restore sweep on the twin: +eps, -2eps, +eps
        for s in (1.0, -2.0, 1.0):
            tr.perturb(named_twin, proj["seed"], s, opt.zo_eps, "normal")
        before = {n: params[n].detach().clone() for n, _ in named_twin}
        captured = capture_ns_outputs(opt)
        st = opt.step()
        steps.append(st)
        if not st["skipped"]:
            torch.cuda.synchronize()
            ref = tr.step(named_twin, list(opt.history), lr=st["lr"], beta=opt.beta_momentum, ns_steps=opt.ns_steps,
                          muon_scale=opt.muon_scale, ratio_clip=opt.update_ratio_clip,
                          weight_decay=opt.weight_decay, distribution="normal")
            assert ref["updated_param_count"] == st["updated_param_count"] == len(captured)
            for n, p in named_twin:
                w0 = before[n]
                w0n = w0.cpu().numpy()
                ideal = exact_block_update(w0, n, 0, list(opt.history), opt, st["lr"], "normal")
                mine = block_update_from_ns(w0, captured[(n, 0)], opt, st["lr"])
                got = params[n].detach().cpu().numpy()
                r_u = rel(mine.u, ideal.u)
                r_stored = rel(got - w0n, ideal.w - w0n)
                r_ref = rel(p.detach().cpu().numpy() - w0n, ideal.w - w0n)
                assert rel(got - w0n, p.detach().cpu().numpy() - w0n) <= r_ref + 2e-2, n
                max_u, max_stored = max(max_u, r_u), max(max_stored, r_stored)
            # keep both on the same weights so each step is compared from a common start
            with torch.no_grad():
                for (n, p) in named_twin:
                    p.copy_(params[n].detach())
    # fp32 weights: every update within 2e-2 of the exact-accumulation iteration's
    print("tiny llama: max update error", round(max_u, 4), "stored", round(max_stored, 4))
    assert max_u <= 2e-2 and max_stored <= 2e-2, (max_u, max_stored)
    losses = [p["loss_plus"] for p in projections]
    assert all(math.isfinite(x) for x in losses)
    used = [p["p_used"] for p in projections if not p["skipped"]]
    assert used and not all(abs(abs(u) - 3.0) < 1e-9 for u in used)          # not glued to +-3
    applied = [s for s in steps if not s["skipped"]]
    assert len(applied) >= 10
    assert all(s["update_ratio_max"] <= opt.update_ratio_clip * (1 + 1e-3) for s in applied)
    assert steps[0]["skip_reason"] == "waiting for min_history=4"
    qk = opt.probe_and_apply_qk_clip(closure, force_eager=True)
    assert qk["enabled"] and qk["exact_logits"] and qk["qk_smax_max"] > 0.0
    assert set(qk) == {"enabled", "exact_logits", "fallback_used", "disabled_reason", "qk_smax_max", "qk_clip_count"}


def _selected(model, opt):
    names = set(opt.selected_parameter_names())
    return {n: p.detach().clone() for n, p in model.named_parameters() if n in names}


def test_restore_exact_and_rollback_restore_bitwise(device):
    """restore_exact replaces the +eps restore pass with the host snapshot (muzo_optimizer.py:208-211)
    and rollback restores it when the projection is rejected (218-221): in bf16 both must give the
    weights back bit for bit, through the page-locked snapshot buffers."""
    from muzo_clip_b200 import MuZOClipOptimizer

    model = _model(device).to(torch.bfloat16)
    ids = torch.randint(0, 1024, (2, 32), generator=torch.Generator().manual_seed(1)).to(device)

    def closure():
        return model(input_ids=ids, labels=ids).loss

    opt = MuZOClipOptimizer(model, restore_exact=True, seed=7)
    for _ in range(2):
        before = _selected(model, opt)
        proj = opt.estimate_projection(closure)
        assert not proj["skipped"]
        after = _selected(model, opt)
        assert all(torch.equal(before[n], after[n]) for n in before)
    assert opt._snapshot_bufs is not None and opt._snapshot_bufs[0].is_pinned()

    calls = {"n": 0}

    def bad_closure():
        calls["n"] += 1
        return float("nan") if calls["n"] == 2 else closure()

    opt = MuZOClipOptimizer(model, rollback=True, seed=9)
    before = _selected(model, opt)
    proj = opt.estimate_projection(bad_closure)
    assert proj["skipped"] and proj["skip_reason"] is not None
    after = _selected(model, opt)
    assert all(torch.equal(before[n], after[n]) for n in before)
    assert not opt.history
