"""Prove tests/golden/torch_reference.py equal to the real reference package, bit for bit.

Runs in the build container only (the reference is mounted there, not on GPU machines), on CPU
tensors: both sides issue the same PyTorch ops, so every result must match exactly. Also writes
tests/golden/hash_kat.json, the reference's own hash64_seed outputs.

Usage: python tests/golden/check_against_reference.py [--reference /root/reference]
"""

from __future__ import annotations

import argparse
import copy
import json
import random
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import torch_reference as tr  # noqa: E402


def _tiny_model(dtype=torch.float32):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      intermediate_size=96, vocab_size=128, attn_implementation="eager")
    return LlamaForCausalLM(cfg).to(dtype)


HASH_CASES = [
    (12345, "model.layers.0.self_attn.q_proj.weight", (4096, 4096), 0),
    (1, "model.layers.31.mlp.down_proj.weight", (4096, 14336), 0),
    (2**63 - 2, "model.layers.7.mlp.gate_proj.weight", (14336, 4096), 3),
    (0, "w", (1, 1), 0),
    (987654321987654321, "model.layers.79.self_attn.k_proj.weight", (1024, 8192), 12),
    (42, "a" * 300, (7, 9), 1),
]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from muzo_clip import MuZOClipOptimizer, zeropower_via_newtonschulz5
    from muzo_clip.muzo_optimizer import HistoryItem
    from muzo_clip.prng import hash64_seed, make_zo_noise_like

    # 1. hash known answers
    kat = []
    for seed, name, shape, bi in HASH_CASES:
        ref = hash64_seed(seed, name, shape, bi)
        assert tr.hash64_seed(seed, name, shape, bi) == ref
        kat.append({"seed": seed, "name": name, "shape": list(shape), "block": bi, "key": ref})
    (HERE / "hash_kat.json").write_text(json.dumps(kat, indent=1) + "\n")

    # 2. noise (CPU generator): same ops, same values
    for dist in ("normal", "rademacher"):
        for dtype in (torch.float32, torch.bfloat16):
            t = torch.zeros((33, 17), dtype=dtype)
            a = make_zo_noise_like(t, 7, "x.weight", 2, dist)
            b = tr.noise_like(t, 7, "x.weight", 2, dist)
            assert torch.equal(a, b), (dist, dtype)

    # 3. Newton-Schulz (CPU path)
    g = torch.Generator().manual_seed(3)
    for shape in ((24, 40), (40, 24)):
        G = torch.randn(shape, generator=g)
        assert torch.equal(zeropower_via_newtonschulz5(G, 5), tr.newton_schulz(G, 5)), shape

    # 4. a full step against the reference optimizer on a tiny Llama (both distributions,
    #    with and without row blocks)
    for dist, block_rows in (("normal", None), ("rademacher", None), ("normal", 40)):
        model = _tiny_model()
        twin = copy.deepcopy(model)
        opt = MuZOClipOptimizer(model, seed=11, distribution=dist, block_rows=block_rows, lr=1e-2,
                                update_ratio_clip=0.05)
        rng = random.Random(5)
        for _ in range(6):
            opt.history.append(HistoryItem(seed=rng.randrange(0, 2**63 - 1), p=rng.uniform(-3, 3), p_raw=0.0,
                                           loss_plus=0.0, loss_minus=0.0))
        opt._has_pending_update = True
        stats = opt.step()
        named = [(n, p) for n, p in twin.named_parameters() if n in set(opt.selected_parameter_names())]
        mine = tr.step(named, list(opt.history), lr=opt.current_lr, beta=opt.beta_momentum, ns_steps=opt.ns_steps,
                       muon_scale=opt.muon_scale, ratio_clip=opt.update_ratio_clip,
                       weight_decay=opt.weight_decay, distribution=dist, block_rows=block_rows)
        for key in ("update_rms_mean", "update_ratio_max", "updated_param_count"):
            assert mine[key] == stats[key], (dist, key, mine[key], stats[key])
        for (n1, p1), (n2, p2) in zip(model.named_parameters(), twin.named_parameters()):
            assert torch.equal(p1, p2), (dist, n1)

        # perturbation sweep
        tr.perturb(named, 99, 1.0, opt.zo_eps, dist, block_rows)
        opt._perturb_selected(99, 1.0)
        for (n1, p1), (n2, p2) in zip(model.named_parameters(), twin.named_parameters()):
            assert torch.equal(p1, p2), (dist, "perturb", n1)
    print("torch_reference matches the reference package on CPU:", len(kat), "hash cases, noise, NS, step, perturb")
    return 0


if __name__ == "__main__":
    sys.exit(main())
