"""Parity at the headline shapes: one full Llama-3-8B layer through step(), Newton-Schulz on the
8192 x 28672 matrix of the standalone sweep, and the QK max logit of one Llama-3-70B layer.

These are the shapes where the step's time goes — 256 x 256 CTA-pair tiles, the atomic tile
scheduler and the mirrored symmetric tiles all at full size — checked against

* the exact-accumulation iteration (``exact_ns.ns5_exact``: the reference's bf16 op sequence of
  muzo_clip/newton_schulz.py:44-58 with float64 GEMMs, run on the GPU), which bounds the update
  at the stated tolerance: relative Frobenius error <= 2e-2 on the applied update dtype(U);
* the reference's own path (``torch_reference.step``: the same torch ops as muzo_optimizer.py:
  315-357, cuBLAS GEMMs), whose own distance to the exact iteration is reported beside it.
"""

from __future__ import annotations

import copy
import math
import random

import numpy as np
import pytest
import torch

import torch_reference as tr
from exact_ns import ns5_exact

pytestmark = pytest.mark.gpu

UPDATE_TOL = 2e-2          # relative Frobenius error of the applied update vs the exact iteration

LLAMA3_8B_LAYER = {
    "self_attn.q_proj": (4096, 4096),
    "self_attn.k_proj": (1024, 4096),
    "self_attn.v_proj": (1024, 4096),
    "self_attn.o_proj": (4096, 4096),
    "mlp.gate_proj": (14336, 4096),
    "mlp.up_proj": (14336, 4096),
    "mlp.down_proj": (4096, 14336),
}


class _Layer(torch.nn.Module):
    """One decoder layer's selected matrices with Hugging Face names, bf16 N(0, 0.02)."""

    def __init__(self, device, seed=0):
        super().__init__()
        g = torch.Generator(device=device).manual_seed(seed)
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList([torch.nn.Module()])
        layer = self.model.layers[0]
        layer.self_attn = torch.nn.Module()
        layer.mlp = torch.nn.Module()
        for name, (r, c) in LLAMA3_8B_LAYER.items():
            owner, leaf = name.split(".")
            w = torch.empty((r, c), dtype=torch.bfloat16, device=device)
            w.normal_(0.0, 0.02, generator=g)
            lin = torch.nn.Module()
            lin.weight = torch.nn.Parameter(w, requires_grad=False)
            setattr(getattr(layer, owner), leaf, lin)


def _rel(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _rel_t(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


def test_llama3_8b_layer_step_against_exact_iteration(device):
    """step() on q/o 4096 x 4096, k/v 1024 x 4096, gate/up 14336 x 4096, down 4096 x 14336 (bf16,
    H = 8, normal noise, lr 2e-3 so that the ratio clip engages), default kernels:

    * the applied update dtype(U) of every matrix is within 2e-2 (relative Frobenius) of the one
      the exact-accumulation iteration gives for the reference's momentum;
    * >= 90 % of the new bf16 weights are bit-equal to the exact iteration's;
    * the apply kernel is the reference's arithmetic: the new weights equal the oracle's
      scale / clip / apply / decay of this build's own Newton-Schulz result (>= 99.9 % bit-equal,
      the rest one bf16 ulp apart: the ratio clip's factor may differ in its last bit because the
      sums of squares are accumulated in another order);
    * the stored update is no further from the exact iteration than the reference's cuBLAS
      path's is, + 2e-2."""
    import muzo_oracle as orc
    from muzo_clip_b200 import MuZOClipOptimizer
    from muzo_clip_b200.muzo_optimizer import HistoryItem

    model = _Layer(device, seed=3)
    twin = copy.deepcopy(model)
    opt = MuZOClipOptimizer(model, horizon=8, min_history=4, beta_momentum=0.9, lr=2e-3, seed=11)
    rng = random.Random(5)
    for _ in range(8):
        opt.history.append(HistoryItem(rng.randrange(0, 2**63 - 1), max(-3.0, min(3.0, rng.gauss(0, 1))),
                                       0.0, 0.0, 0.0))
    opt._has_pending_update = True
    names = opt.selected_parameter_names()
    assert len(names) == 7
    params = dict(model.named_parameters())
    before = {n: params[n].detach().clone() for n in names}

    captured: dict[str, torch.Tensor] = {}

    def hook(blocks, x, stream):
        with torch.cuda.stream(stream):
            for j, b in enumerate(blocks):
                captured[b.name] = x[j].clone()

    eng = opt._engine_for_step()
    eng.ns_output_hook = hook
    stats = opt.step()
    torch.cuda.synchronize()
    assert not stats["skipped"] and stats["updated_param_count"] == 7
    assert set(captured) == set(names)

    named_twin = [(n, p) for n, p in twin.named_parameters() if n in set(names)]
    ref_stats = tr.step(named_twin, list(opt.history), lr=stats["lr"], beta=opt.beta_momentum,
                        ns_steps=opt.ns_steps, muon_scale=opt.muon_scale, ratio_clip=opt.update_ratio_clip,
                        weight_decay=opt.weight_decay, distribution="normal")
    assert ref_stats["updated_param_count"] == 7
    twin_params = dict(twin.named_parameters())

    report = {}
    exact_ratios, exact_rms = [], []
    for name in names:
        w0 = before[name]
        M = tr.rebuild(w0, name, 0, list(opt.history), opt.beta_momentum, "normal", True)
        x_exact = ns5_exact(M, opt.ns_steps)
        x_mine = captured[name].float()
        del M
        w0n = w0.float().cpu().numpy()
        res_exact = orc.apply_update(w0n, x_exact.cpu().numpy(), stats["lr"], opt.muon_scale, opt.update_ratio_clip,
                                     opt.weight_decay, "bf16")
        res_mine = orc.apply_update(w0n, x_mine.cpu().numpy(), stats["lr"], opt.muon_scale, opt.update_ratio_clip,
                                    opt.weight_decay, "bf16")
        exact_ratios.append(res_exact.ratio)
        exact_rms.append(res_exact.update_rms)
        mine_w = params[name].detach().float().cpu().numpy()
        ref_w = twin_params[name].detach().float().cpu().numpy()
        r_u = _rel(res_mine.u, res_exact.u)
        r_x = _rel_t(x_mine, x_exact)
        same_exact = float(np.mean(mine_w == res_exact.w))
        same_apply = float(np.mean(mine_w == res_mine.w))
        ulp = np.abs(res_mine.w) * 2.0 ** -7 + 1e-30
        apply_gap = float(np.max(np.abs(mine_w - res_mine.w) / ulp))
        r_mine = _rel(mine_w - w0n, res_exact.w - w0n)
        r_ref = _rel(ref_w - w0n, res_exact.w - w0n)
        report[name] = dict(u=round(r_u, 4), x=round(r_x, 4), bit_equal_exact=round(same_exact, 4),
                            bit_equal_apply=round(same_apply, 5), stored_mine=round(r_mine, 4),
                            stored_ref=round(r_ref, 4), clipped=res_exact.clipped)
        print(name, report[name])
        assert r_u <= UPDATE_TOL, (name, report[name])
        assert same_exact >= 0.9, (name, report[name])
        assert same_apply >= 0.999 and apply_gap <= 1.0 + 1e-6, (name, report[name], apply_gap)
        assert r_mine <= r_ref + 2e-2, (name, report[name])
    # step statistics against the exact iteration's
    assert abs(stats["update_ratio_max"] - max(exact_ratios)) <= UPDATE_TOL * max(exact_ratios)
    mean_rms = sum(exact_rms) / len(exact_rms)
    assert abs(stats["update_rms_mean"] - mean_rms) <= UPDATE_TOL * mean_rms
    assert any(r["clipped"] for r in report.values())


def test_newton_schulz_8192x28672_against_exact_iteration(device):
    """zeropower_via_newtonschulz5 on the largest matrix of the standalone Newton-Schulz sweep
    (8192 x 28672, fp32 N(0, 1)): within 2e-2 of the exact-accumulation iteration, and no further
    from the reference's cuBLAS result than that result is from the exact iteration, + 2e-2."""
    from muzo_clip_b200 import zeropower_via_newtonschulz5

    g = torch.Generator(device=device).manual_seed(8192)
    G = torch.randn((8192, 28672), generator=g, device=device)
    mine = zeropower_via_newtonschulz5(G, 5)
    exact = ns5_exact(G, 5)
    r_mine = _rel_t(mine, exact)
    ref = tr.newton_schulz(G, 5)
    r_ref = _rel_t(ref, exact)
    print("8192x28672", dict(mine=round(r_mine, 4), ref=round(r_ref, 4), mine_vs_ref=round(_rel_t(mine, ref), 4)))
    assert mine.dtype == torch.float32 and mine.shape == G.shape
    assert r_mine <= UPDATE_TOL, (r_mine, r_ref)
    assert _rel_t(mine, ref) <= r_ref + 2e-2


def test_qk_max_llama3_70b_layer(device):
    """Per-head max logit of one Llama-3-70B-shaped attention layer (B = 1, S = 4096, 64 query /
    8 KV heads of dim 128, causal, bf16 N(0, 1) post-RoPE states in transformers' [B, S, H, D]
    layout) against eager attention's pre-softmax logits: within one bf16 ulp per head."""
    from muzo_clip_b200 import _qk

    g = torch.Generator(device=device).manual_seed(70)
    q = torch.randn((1, 4096, 64, 128), generator=g, device=device).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn((1, 4096, 8, 128), generator=g, device=device).to(torch.bfloat16).transpose(1, 2)
    scale = 128 ** -0.5
    got, valid = _qk.qk_head_max(q, k, scale, True, None)
    torch.cuda.synchronize()
    assert int(valid.item()) == 1
    want = tr.qk_head_max(tr.eager_logits(q, k, scale, True))
    got = got.cpu()
    ulp = torch.pow(2.0, torch.floor(torch.log2(want.abs().clamp_min(2.0 ** -126))) - 7)
    assert bool(((got - want).abs() <= ulp).all()), (got, want)
    assert math.isfinite(float(got.max()))
