"""Prove oracle/torch_reference.py equal to the real reference package, bit for bit — TEST
INFRASTRUCTURE.

Both sides issue the same PyTorch ops, so every result must match exactly on the same device:
``check_all(device)`` runs the comparisons (hash64_seed, make_zo_noise_like, the Newton-Schulz
iteration, a full step and a perturbation sweep through the reference's own optimizer).
``tests/test_reference_link_cpu.py`` runs them on CPU tensors (the reference's fp32 branch of
newton_schulz.py:46) and ``tests/test_reference_link_gpu.py`` on CUDA tensors (its bf16 branch,
cuBLAS), wherever the reference package can be imported (``reference_pkg``). As a script it also
writes tests/golden/hash_kat.json, the reference's own hash64_seed outputs.

Usage: python tests/golden/check_against_reference.py [--reference DIR] [--device cpu|cuda]
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
sys.path.insert(0, str(HERE.parents[1] / "oracle"))

import torch_reference as tr  # noqa: E402

HASH_CASES = [
    (12345, "model.layers.0.self_attn.q_proj.weight", (4096, 4096), 0),
    (1, "model.layers.31.mlp.down_proj.weight", (4096, 14336), 0),
    (2**63 - 2, "model.layers.7.mlp.gate_proj.weight", (14336, 4096), 3),
    (0, "w", (1, 1), 0),
    (987654321987654321, "model.layers.79.self_attn.k_proj.weight", (1024, 8192), 12),
    (42, "a" * 300, (7, 9), 1),
]


def _tiny_model(device, dtype=torch.float32):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      intermediate_size=96, vocab_size=128, attn_implementation="eager")
    return LlamaForCausalLM(cfg).to(dtype).to(device)


def hash_kat(ref) -> list[dict]:
    """The reference's hash64_seed on HASH_CASES, checked against the restatement."""
    kat = []
    for seed, name, shape, bi in HASH_CASES:
        key = ref.prng.hash64_seed(seed, name, shape, bi)
        assert tr.hash64_seed(seed, name, shape, bi) == key
        kat.append({"seed": seed, "name": name, "shape": list(shape), "block": bi, "key": key})
    return kat


def check_noise(ref, device) -> None:
    for dist in ("normal", "rademacher"):
        for dtype in (torch.float32, torch.bfloat16, torch.float16):
            for shape in ((33, 17), (1000, 1031)):
                t = torch.zeros(shape, dtype=dtype, device=device)
                a = ref.prng.make_zo_noise_like(t, 7, "x.weight", 2, dist)
                b = tr.noise_like(t, 7, "x.weight", 2, dist)
                assert torch.equal(a, b), (dist, dtype, shape)


def check_newton_schulz(ref, device) -> None:
    g = torch.Generator(device="cpu").manual_seed(3)
    for shape in ((24, 40), (40, 24), (256, 688), (688, 256)):
        G = torch.randn(shape, generator=g).to(device)
        for steps in (0, 1, 5):
            a = ref.newton_schulz.zeropower_via_newtonschulz5(G, steps)
            assert torch.equal(a, tr.newton_schulz(G, steps)), (shape, steps)
    z = torch.zeros((16, 16), device=device)
    assert torch.equal(ref.newton_schulz.zeropower_via_newtonschulz5(z), tr.newton_schulz(z))


def check_step_and_perturb(ref, device, dtype=torch.float32) -> None:
    """A full step() of the reference optimizer on a tiny Llama against torch_reference.step on a
    twin (both distributions, with and without row blocks), then a perturbation sweep."""
    from muzo_clip.muzo_optimizer import HistoryItem

    for dist, block_rows in (("normal", None), ("rademacher", None), ("normal", 40)):
        model = _tiny_model(device, dtype)
        twin = copy.deepcopy(model)
        opt = ref.MuZOClipOptimizer(model, seed=11, distribution=dist, block_rows=block_rows, lr=1e-2,
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
        tr.perturb(named, 99, 1.0, opt.zo_eps, dist, block_rows)
        opt._perturb_selected(99, 1.0)
        for (n1, p1), (n2, p2) in zip(model.named_parameters(), twin.named_parameters()):
            assert torch.equal(p1, p2), (dist, "perturb", n1)


def main() -> int:
    from reference_pkg import reference_path

    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="directory holding the muzo_clip package")
    ap.add_argument("--device", default="cpu")
    args = ap.parse_args()
    root = args.reference or reference_path()
    if root is None:
        raise SystemExit("reference package not found: pass --reference or set MUZO_REFERENCE_PATH")
    sys.path.insert(0, str(root))
    import muzo_clip as ref
    import muzo_clip.newton_schulz  # noqa: F401
    import muzo_clip.prng  # noqa: F401

    device = torch.device(args.device)
    kat = hash_kat(ref)
    (HERE / "hash_kat.json").write_text(json.dumps(kat, indent=1) + "\n")
    check_noise(ref, device)
    check_newton_schulz(ref, device)
    check_step_and_perturb(ref, device)
    print("torch_reference matches the reference package on", device, ":", len(kat), "hash cases, noise, NS, step, perturb")
    return 0


if __name__ == "__main__":
    sys.exit(main())
