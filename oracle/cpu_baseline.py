"""CPU baseline of the optimizer step on the host cores — BENCHMARK INFRASTRUCTURE ONLY.

Runs the reference's own op sequence (``torch_reference``: the torch ops of
muzo_clip/muzo_optimizer.py:190-357 and newton_schulz.py:17-66, in the same order and dtypes) on
CPU tensors with all the host threads torch may use, one Llama-3-8B matrix at a time: three
perturbation passes (+eps, -2eps, +eps), the H = 8 normal-noise momentum rebuild, Newton-Schulz
(the reference's CPU branch: fp32) and the scale / clip / apply / decay update. The step of the
whole model is extrapolated from one matrix of each of the four shape classes (per layer: two
4096 x 4096, two 1024 x 4096, two 14336 x 4096 and one 4096 x 14336), by count. Only
``bench.py`` uses it, for its reported CPU baseline and its reference arm.
"""

from __future__ import annotations

import os
import random
import time

import torch

import torch_reference as tr

# (rows, cols), a parameter name of that shape, matrices of the class per decoder layer
CLASSES = (
    ((1024, 4096), "model.layers.0.self_attn.k_proj.weight", 2),
    ((4096, 4096), "model.layers.0.self_attn.q_proj.weight", 2),
    ((14336, 4096), "model.layers.0.mlp.gate_proj.weight", 2),
    ((4096, 14336), "model.layers.0.mlp.down_proj.weight", 1),
)
LAYERS = 32
HORIZON = 8


class _Item:
    def __init__(self, seed: int, p: float):
        self.seed, self.p = seed, p


def host_threads() -> int:
    """Host threads this process may run on; torch's intra-op pool is set to that many."""
    try:
        n = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        n = os.cpu_count() or 1
    return max(1, n)


def use_all_threads() -> int:
    torch.set_num_threads(host_threads())
    return torch.get_num_threads()


@torch.no_grad()
def matrix_step(cls: int, seed: int = 0) -> tuple[float, float, float, float]:
    """Seconds spent on one bf16 matrix of shape class `cls` in (perturbation passes, rebuild,
    Newton-Schulz, update)."""
    (rows, cols), name, _ = CLASSES[cls]
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn((rows, cols), generator=g) * 0.02).to(torch.bfloat16)
    rng = random.Random(seed)
    hist = [_Item(rng.randrange(0, 2**63 - 1), max(-3.0, min(3.0, rng.gauss(0, 1)))) for _ in range(HORIZON)]
    pseed = rng.randrange(0, 2**63 - 1)
    named = [(name, w)]
    t0 = time.perf_counter()
    for s in (1.0, -2.0, 1.0):
        tr.perturb(named, pseed, s, 1e-3, "normal")
    t1 = time.perf_counter()
    M = tr.rebuild(w, name, 0, hist, 0.9, "normal", True)
    t2 = time.perf_counter()
    U = tr.newton_schulz(M, 5)
    t3 = time.perf_counter()
    tr.apply_update(w, U, 1e-5, 0.2, 0.01, 0.01)
    t4 = time.perf_counter()
    return t1 - t0, t2 - t1, t3 - t2, t4 - t3


def step_ms(seconds_by_class: dict[int, float]) -> float:
    """Milliseconds of the whole 224-matrix step from one matrix's seconds per class."""
    return 1e3 * LAYERS * sum(CLASSES[c][2] * s for c, s in seconds_by_class.items())


def describe(samples: dict[int, list[float]], threads: int) -> str:
    parts = []
    for c, times in sorted(samples.items()):
        (r, k), _, n = CLASSES[c]
        parts.append(f"{r}x{k}: {len(times)} x {min(times):.1f}-{max(times):.1f} s (x{n * LAYERS})")
    return (f"the reference's torch op sequence on CPU tensors, {threads} torch threads (nproc "
            f"{os.cpu_count()}): one bf16 matrix per sample through 3 perturbation passes, the H=8 "
            f"normal-noise rebuild, fp32 Newton-Schulz (the reference's CPU branch) and the update; "
            f"{'; '.join(parts)}; the 224-matrix step extrapolated by count from each class's median")


@torch.no_grad()
def ns_seconds(rows: int, cols: int, seed: int = 0) -> float:
    """Seconds of the reference's Newton-Schulz (five iterations, its CPU branch: fp32) on one
    fp32 N(0, 1) matrix of rows x cols (the sweep of configuration 3 times one matrix per shape)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((rows, cols), generator=g)
    t0 = time.perf_counter()
    tr.newton_schulz(x, 5)
    return time.perf_counter() - t0


@torch.no_grad()
def perturb_pass_seconds(numel: int, dist: str = "rademacher", seed: int = 0) -> float:
    """Seconds of one perturbation pass of the reference's op sequence (noise generated on the
    CPU, W <- bf16(W + eps * Z)) over a flat bf16 tensor [numel / 4096, 4096]."""
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn((numel // 4096, 4096), generator=g) * 0.02).to(torch.bfloat16)
    named = [("model.layers.0.mlp.up_proj.weight", w)]
    t0 = time.perf_counter()
    tr.perturb(named, 12345 + seed, 1.0, 1e-3, dist)
    return time.perf_counter() - t0
