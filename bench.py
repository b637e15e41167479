"""Benchmark of the MuZO-Clip optimizer step on Llama-3-8B-shaped matrices.

One step = the optimizer share of ``estimate_projection`` (three perturbation passes: +eps,
-2eps, +eps, over every selected matrix; the loss closure returns synthetic scalars, no model
forward) followed by ``step()`` (H=8 momentum rebuild, Newton-Schulz, scaled/clipped update with
weight decay) through the public MuZOClipOptimizer API. The history is filled by H projections
before the warm-up, as in a running job. The line reports the optimizer with noise_cache=True
(each projection's rounded noise kept on the device, bit-identical results); the default
configuration, which regenerates all noise, is timed in the same run under "variants".

Workload: 32 layers x {q 4096x4096, k 1024x4096, v 1024x4096, o 4096x4096, gate 14336x4096,
up 14336x4096, down 4096x14336}, bf16 N(0, 0.02) weights, horizon 8, beta 0.9, p ~ N(0,1) clipped
to +-3, random 63-bit seeds. Synthetic data; 14 GB of weights, far larger than L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 runs under torchrun: every rank holds a replica, perturbs it locally, and rebuilds /
orthogonalises / applies the matrices it owns (LPT partition by Newton-Schulz FLOPs); the owners
push the updated weights into the other ranks' replicas. ``--impl reference`` times the
reference's op sequence on CPU tensors (one matrix per timed step, the four shape classes in
turn) on the host cores, extrapolated to the full step.

``--workload llama3-70b`` times the Llama-3-70B-shaped case instead (80 layers of q/o 8192x8192,
k/v 1024x8192, gate/up 28672x8192, down 8192x28672: 68.4 G bf16 weights, 137 GB per replica, so
no noise pool fits next to them): the same step with regenerated noise, then the QK-Clip probe
over 80 layers (per-head max logit of synthetic Q [1, 64, 4096, 128] and K [1, 8, 4096, 128]
activations per layer, causal, the maxima max-reduced over the ranks, the q/k rows scaled) through
the optimizer's QK-Clip controller, without a model forward.
"""

from __future__ import annotations

import argparse
import gc
import json
import math
import os
import random
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "muzo-clip_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

LAYERS = 32
HIDDEN = 4096
KV = 1024
MLP = 14336
SHAPES = {
    "self_attn.q_proj": (HIDDEN, HIDDEN),
    "self_attn.k_proj": (KV, HIDDEN),
    "self_attn.v_proj": (KV, HIDDEN),
    "self_attn.o_proj": (HIDDEN, HIDDEN),
    "mlp.gate_proj": (MLP, HIDDEN),
    "mlp.up_proj": (MLP, HIDDEN),
    "mlp.down_proj": (HIDDEN, MLP),
}
SHAPES_70B = {
    "self_attn.q_proj": (8192, 8192),
    "self_attn.k_proj": (1024, 8192),
    "self_attn.v_proj": (1024, 8192),
    "self_attn.o_proj": (8192, 8192),
    "mlp.gate_proj": (28672, 8192),
    "mlp.up_proj": (28672, 8192),
    "mlp.down_proj": (8192, 28672),
}
LAYERS_70B = 80
HORIZON = 8
METRIC = "MuZO step() ms & perturb HBM GB/s, Llama-3-8B shapes, 1/2/4/8 B200"
WORKLOAD = "llama3-8b-selected-matrices"


def total_numel(layers: int = LAYERS) -> int:
    return layers * sum(r * c for r, c in SHAPES.values())


def ns_flops_total(layers: int = LAYERS, steps: int = 5) -> float:
    tot = 0.0
    for r, c in SHAPES.values():
        m, n = min(r, c), max(r, c)
        tot += steps * (4.0 * m * m * n + 2.0 * m ** 3)
    return layers * tot


class Llama8BMatrices(torch.nn.Module):
    """Selected-parameter skeleton of a Llama model with HF names (no forward): Llama-3-8B
    shapes unless ``shapes`` names others."""

    def __init__(self, device, dtype=torch.bfloat16, layers: int = LAYERS, seed: int = 0,
                 shapes: dict | None = None):
        super().__init__()
        shapes = SHAPES if shapes is None else shapes
        g = torch.Generator(device=device).manual_seed(seed)
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList()
        for _ in range(layers):
            layer = torch.nn.Module()
            layer.self_attn = torch.nn.Module()
            layer.mlp = torch.nn.Module()
            for name, (r, c) in shapes.items():
                owner, leaf = name.split(".")
                w = torch.empty((r, c), dtype=dtype, device=device)
                w.normal_(0.0, 0.02, generator=g)
                lin = torch.nn.Module()
                lin.weight = torch.nn.Parameter(w, requires_grad=False)
                setattr(getattr(layer, owner), leaf, lin)
            self.model.layers.append(layer)


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"muzo_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi takes a moment to start: wait (at most 3 s) for its first sample, so that a
        # short timed region (a few steps of ~100 ms on 8 GPUs) is still sampled
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < 3.0 and self.proc.poll() is None:
            try:
                if self.path.stat().st_size > 0:
                    break
            except OSError:
                pass
            time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = [l.split(",") for l in self.path.read_text().strip().splitlines() if l.strip()]
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        try:
            self.path.unlink()
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# DRAM traffic measured by one ncu capture of this workload on one B200 (1-pass metrics
# gpu__time_duration.sum, dram__bytes_read.sum, dram__bytes_write.sum, --clock-control none, on
# `python bench.py --steps 1 --warmup 1 --no-cpu-baseline --no-variant`): read + write of the
# timed step, summed over its 105 ns_gemm launches, per perturbation pass and for the rebuild.
NS_DRAM_BYTES_PER_STEP = 462.2e9
PERTURB_DRAM_BYTES_PER_PASS = 27.89e9          # a pass that regenerates its noise
PERTURB_KEPT_DRAM_BYTES_PER_PASS = 41.92e9     # mean of the keeping pass and the two kept passes
REBUILD_KEPT_DRAM_BYTES_PER_STEP = 139.52e9
TRAFFIC_SOURCE = "profiles/launches_dram_llama3_8b_step.md (one ncu capture, not measured in this run)"


def ns_operand_bytes(rows: int, cols: int, steps: int = 5) -> float:
    """Minimal DRAM bytes of the Newton-Schulz GEMMs for one matrix: per iteration X read and A
    written (X X^T), A read and B written (b A + c A A), B and X read and X written (a X + B X),
    each once: 6 m n + 8 m^2 bytes in bf16, m = min(rows, cols), n = max."""
    m, n = min(rows, cols), max(rows, cols)
    return steps * (6.0 * m * n + 8.0 * m * m)


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------- CPU baseline


def _cpu_baseline_module():
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_baseline

    return cpu_baseline


def cpu_sample_ms(seed: int = 0) -> tuple[float, str, int]:
    """The reference's op sequence on CPU tensors, one matrix of each of the four shape classes
    (all host threads), extrapolated to the 224-matrix step."""
    cb = _cpu_baseline_module()
    threads = cb.use_all_threads()
    samples = {c: [sum(cb.matrix_step(c, seed + c))] for c in range(len(cb.CLASSES))}
    ms = cb.step_ms({c: statistics.median(v) for c, v in samples.items()})
    return ms, cb.describe(samples, threads), threads


# ---------------------------------------------------------------- GPU arm


def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        # a rank that stops answering ends the others' next collective with an error
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
        return dist, rank, world, local
    torch.cuda.set_device(local)
    return None, 0, 1, local


def _time_steps(opt, args, device, dist, local) -> dict:
    """Fill the history through H projections and steps, run W warm-up steps, then time exactly K
    steps (estimate_projection + step) with CUDA events on the launching stream between a barrier
    and a synchronize on both sides, max over ranks; per-phase device time from CUDA events, wall
    time through the public API, nvidia-smi clocks sampled during the timed steps."""
    from muzo_clip_b200 import _lib

    loss_rng = random.Random(7)

    def closure():
        return 2.0 + 0.01 * loss_rng.random()

    def one_step():
        opt.estimate_projection(closure)
        return opt.step()

    # optimizer state of a running job: a full history, each entry made by a projection
    for _ in range(HORIZON):
        one_step()
    for _ in range(args.warmup):
        st = one_step()
        assert not st["skipped"], st
    stream = torch.cuda.current_stream(device)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    engine = opt._engine
    barrier()
    launches0 = _lib.launch_count
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    engine.start_phase_timing()
    with ClockSampler(local) as clocks:
        w0 = time.perf_counter()
        start.record(stream)
        for _ in range(args.steps):
            one_step()
        end.record(stream)
        barrier()
        w1 = time.perf_counter()
    phases = {k: v / args.steps for k, v in engine.stop_phase_timing().items()}
    launches = _lib.launch_count - launches0
    dev_ms = start.elapsed_time(end) / args.steps
    wall_ms = (w1 - w0) * 1e3 / args.steps
    if dist is not None:
        t = torch.tensor([dev_ms, wall_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, wall_ms = t.tolist()
    return {"dev_ms": dev_ms, "wall_ms": wall_ms, "phases": phases, "launches": launches, "clocks": clocks.summary(),
            "kept_entries": engine.kept_entries, "noise_slots": len(engine.slot_seed),
            "keep_noise": bool(engine.keep_noise)}


def run_gpu(args) -> int:
    dist, rank, world, local = setup_dist()
    device = torch.device("cuda", local)
    from muzo_clip_b200 import MuZOClipOptimizer

    model = Llama8BMatrices(device, layers=args.layers)
    pg = dist.group.WORLD if dist is not None else None

    def make(noise_cache):
        return MuZOClipOptimizer(model, horizon=HORIZON, min_history=4, beta_momentum=0.9, lr=1e-5, seed=1234,
                                 process_group=pg, noise_cache=noise_cache)

    # the configuration the line reports (the noise of the current projection and of every
    # history entry kept in device memory; bit-identical results), then, as a variant, the
    # optimizer's default configuration (every pass and the rebuild regenerate the noise)
    opt = make(not args.no_noise_cache)
    run = _time_steps(opt, args, device, dist, local)
    engine = opt._engine
    phases, dev_ms, wall_ms = run["phases"], run["dev_ms"], run["wall_ms"]
    variant = None
    if not args.no_variant and not args.no_noise_cache:
        noise_pool = engine.noise_pool
        engine.noise_pool = None
        del noise_pool
        torch.cuda.empty_cache()
        plain = make(False)
        variant = _time_steps(plain, args, device, dist, local)
        del plain
        gc.collect()    # the optimizer and its engine reference each other
        torch.cuda.empty_cache()

    n_elems = total_numel(args.layers)
    kept = run["keep_noise"] and run["kept_entries"] == HORIZON
    perturb_ms = phases.get("perturb", 0.0) / 3.0          # three passes per step
    perturb_bytes = 4.0 * n_elems                          # per pass, algorithmic
    perturb_gbs = perturb_bytes / (perturb_ms * 1e-3) / 1e9 if perturb_ms > 0 else 0.0
    # moved per step by the three passes: W read and written each pass, plus the noise written
    # once and read twice when it is kept
    perturb_moved = (3 * 4.0 + (3 * 2.0 if run["keep_noise"] else 0.0)) * n_elems
    ns_ms = phases.get("ns", 0.0)
    ns_flops = engine.owned_ns_flops()
    ns_exec = engine.owned_ns_flops_executed()
    ns_tflops = ns_flops / (ns_ms * 1e-3) / 1e12 if ns_ms > 0 else 0.0
    ns_exec_tflops = ns_exec / (ns_ms * 1e-3) / 1e12 if ns_ms > 0 else 0.0

    # Rademacher perturbation bandwidth (untimed, after the timed region): one pass over the
    # same matrices through an optimizer configured for Rademacher noise
    del opt
    gc.collect()
    torch.cuda.empty_cache()
    rad = MuZOClipOptimizer(model, distribution="rademacher", seed=4321)
    rad_engine = rad._engine_for_step()
    for _ in range(3):
        rad_engine.perturb(777, 1e-3)
    torch.cuda.synchronize()
    rad_engine.start_phase_timing()
    for _ in range(4):
        rad_engine.perturb(777, 1e-3)
        rad_engine.perturb(777, -1e-3)
    rad_ms = rad_engine.stop_phase_timing().get("perturb", 0.0) / 8.0
    rad_gbs = perturb_bytes / (rad_ms * 1e-3) / 1e9 if rad_ms > 0 else 0.0

    if rank == 0:
        peaks = load_peaks()
        hbm = peaks["hbm_gbs"]
        ns_bytes_min = sum(ns_operand_bytes(b.rows, b.cols) for b in engine.owned)
        owned_elems = sum(b.rows * b.cols for b in engine.owned)
        rebuild_ms = max(phases.get("rebuild", 0.0), 1e-9)
        rebuild_bytes = 4.0 * owned_elems                  # bf16(M) written, W read
        apply_ms = max(phases.get("apply", 0.0), 1e-9)
        apply_bytes = 6.0 * owned_elems        # update read (bf16), W read, W written
        norm_ms = max(phases.get("normalize", 0.0), 1e-9)
        norm_bytes = 4.0 * owned_elems         # bf16 momentum read and written
        h2d = 8 * len(engine.blocks) * 3 + 8 * len(engine.owned) * HORIZON + 12 * HORIZON
        d2h = getattr(engine, "g_bytes", engine.state_bytes) + 16

        def gbs(nbytes, ms):
            return round(nbytes / (ms * 1e-3) / 1e9, 1)

        if kept:
            # every history entry read from its kept noise: H bf16 reads, W read, bf16(M) written
            moved = (2.0 * HORIZON + 4.0) * owned_elems
            rebuild_roofline = {
                "bound": "hbm", "kernel": "rebuild_kept_linear_kernel", "achieved": gbs(moved, rebuild_ms),
                "unit": "GB/s", "peak": hbm, "frac": round(gbs(moved, rebuild_ms) / hbm, 4),
                "bytes": moved, "bytes_note": "2H + 4 B per weight actually moved (H kept noise entries read)",
                "traffic": REBUILD_KEPT_DRAM_BYTES_PER_STEP if world == 1 else None, "traffic_source": TRAFFIC_SOURCE,
                "algorithmic_bytes": rebuild_bytes, "algorithmic_achieved": gbs(rebuild_bytes, rebuild_ms),
                "algorithmic_frac": round(gbs(rebuild_bytes, rebuild_ms) / hbm, 4)}
        else:
            # the rebuild regenerates H normal samples per weight: bound by the instruction issue
            # rate (ncu: 43 instructions per sample, 74 % issue utilisation), not by HBM
            rebuild_roofline = {
                "bound": "issue", "kernel": "rebuild_kernel",
                "achieved": round(float(HORIZON) * owned_elems / (rebuild_ms * 1e-3) / 1e9, 1),
                "unit": "G normal samples/s", "hbm_achieved": gbs(rebuild_bytes, rebuild_ms),
                "hbm_frac": round(gbs(rebuild_bytes, rebuild_ms) / hbm, 4), "algorithmic_bytes": rebuild_bytes}
        line = {
            "metric": METRIC,
            "value": round(dev_ms, 3),
            "unit": "ms/step",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_ms, 3),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random-init bf16 weights of the named shapes, synthetic SPSA losses)",
            "config": {"workload": WORKLOAD, "layers": args.layers, "matrices": len(engine.blocks),
                       "elements": n_elems, "horizon": HORIZON, "ns_steps": 5, "distribution": "normal",
                       "parallelism": f"replica perturb + NS partition x{world}",
                       "noise_cache": run["keep_noise"], "noise_slots": run["noise_slots"],
                       "kept_history_entries": run["kept_entries"],
                       "history": f"filled by {HORIZON} projections before the warm-up",
                       "l2": "inputs larger than L2 (14 GB of weights per pass)"},
            "perturb_gbs": round(perturb_gbs, 1),
            "perturb_ms": round(perturb_ms, 3),
            "perturb_gbs_rademacher": round(rad_gbs, 1),
            "phase_ms": {k: round(v, 3) for k, v in phases.items()},
            "other_ms": round(dev_ms - sum(phases.values()), 3),
            "ns_tflops": round(ns_tflops, 1),
            "roofline": {
                "bound": "tensor",
                "kernel": "ns_gemm_wide_kernel / ns_gemm_kernel (Newton-Schulz GEMMs; all launches of the timed steps)",
                "achieved": round(ns_tflops, 1),
                "peak": peaks["bf16_tflops_sustained"],
                "unit": "TFLOP/s",
                "frac": round(ns_tflops / peaks["bf16_tflops_sustained"], 4),
                "flops": "dense 5*(4m^2n+2m^3) per matrix; symmetric tiles execute fewer",
                "executed_tflops": round(ns_exec_tflops, 1),
                "executed_frac": round(ns_exec_tflops / peaks["bf16_tflops_sustained"], 4),
                "peak_source": f"{peaks['source']} bf16 sustained",
                "traffic": NS_DRAM_BYTES_PER_STEP if world == 1 else None,
                "traffic_unit": "DRAM bytes per step, all ns_gemm launches",
                "traffic_source": TRAFFIC_SOURCE,
                "operand_bytes": round(ns_bytes_min),
            },
            "perturb_roofline": {
                "bound": "hbm", "achieved": round(perturb_gbs, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(perturb_gbs / hbm, 4), "peak_source": f"{peaks['source']} copy",
                "achieved_note": "4 B per weight and pass (W read + written) over the mean pass time",
                "moved_gbs": gbs(perturb_moved, 3.0 * perturb_ms),
                "moved_frac": round(gbs(perturb_moved, 3.0 * perturb_ms) / hbm, 4),
                "rademacher_achieved": round(rad_gbs, 1), "rademacher_frac": round(rad_gbs / hbm, 4),
                "traffic": PERTURB_KEPT_DRAM_BYTES_PER_PASS if run["keep_noise"] else PERTURB_DRAM_BYTES_PER_PASS,
                "traffic_unit": "DRAM bytes per pass (mean of the step's three)",
                "traffic_source": TRAFFIC_SOURCE, "algorithmic_bytes": perturb_bytes,
            },
            "rebuild_roofline": rebuild_roofline,
            # the apply (update and W read, W written: 6 B per owned weight; the update's sum of
            # squares comes from the last Newton-Schulz GEMM's epilogue) and, separately, the
            # normalisation of the rebuilt momentum (4 B per owned weight)
            "update_roofline": {
                "bound": "hbm", "kernel": "apply_update_kernel", "achieved": gbs(apply_bytes, apply_ms),
                "unit": "GB/s", "peak": hbm, "frac": round(gbs(apply_bytes, apply_ms) / hbm, 4),
                "algorithmic_bytes": apply_bytes,
            },
            "normalize_roofline": {
                "bound": "hbm", "kernel": "ns_normalize_kernel", "achieved": gbs(norm_bytes, norm_ms),
                "unit": "GB/s", "peak": hbm, "frac": round(gbs(norm_bytes, norm_ms) / hbm, 4),
                "algorithmic_bytes": norm_bytes,
            },
            "e2e": {"value": round(wall_ms, 3), "unit": "ms/step", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": int(run["launches"]),
            "clocks": run["clocks"],
        }
        if variant is not None:
            line["variants"] = {"regenerated_noise": {
                "note": "the optimizer's default configuration (noise_cache=False): every pass and history entry "
                        "regenerated from its seed; same workload, timed in this run after the line's own steps",
                "ms_per_step": round(variant["dev_ms"], 3), "e2e_ms_per_step": round(variant["wall_ms"], 3),
                "phase_ms": {k: round(v, 3) for k, v in variant["phases"].items()},
                "gpu_launches": int(variant["launches"]), "clocks": variant["clocks"]}}
        if world == 1 and not args.no_cpu_baseline:
            cpu_ms, sample, cores = cpu_sample_ms()
            line["cpu_baseline"] = {"value": round(cpu_ms, 1), "unit": "ms/step", "cores": cores, "kind": "port",
                                    "sample": sample}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_70b(args) -> int:
    """The Llama-3-70B-shaped step (regenerated noise) and the 80-layer QK-Clip probe."""
    dist, rank, world, local = setup_dist()
    device = torch.device("cuda", local)
    from muzo_clip_b200 import MuZOClipOptimizer

    layers = args.layers if args.layers is not None else LAYERS_70B
    model = Llama8BMatrices(device, layers=layers, shapes=SHAPES_70B)
    pg = dist.group.WORLD if dist is not None else None
    opt = MuZOClipOptimizer(model, horizon=HORIZON, min_history=4, beta_momentum=0.9, lr=1e-5, seed=1234,
                            process_group=pg, noise_cache=False, enable_qk_clip=True, qk_clip_tau=10.0)
    run = _time_steps(opt, args, device, dist, local)
    engine = opt._engine
    phases, dev_ms = run["phases"], run["dev_ms"]
    ns_ms = phases.get("ns", 0.0)
    ns_tflops = engine.owned_ns_flops() / (ns_ms * 1e-3) / 1e12 if ns_ms > 0 else 0.0
    ns_exec_tflops = engine.owned_ns_flops_executed() / (ns_ms * 1e-3) / 1e12 if ns_ms > 0 else 0.0

    # QK-Clip probe: every rank captures its own batch's maxima (here synthetic activations),
    # the controller max-reduces them over the group and scales the q/k rows
    seq, hq, hkv, hd = 4096, 64, 8, 128
    g = torch.Generator(device=device).manual_seed(100 + rank)
    acts = []
    for _ in range(layers):
        q = (torch.randn((1, seq, hq, hd), generator=g, device=device, dtype=torch.bfloat16) * 1.5).transpose(1, 2)
        k = (torch.randn((1, seq, hkv, hd), generator=g, device=device, dtype=torch.bfloat16) * 1.5).transpose(1, 2)
        acts.append((q, k))
    attn = [layer.self_attn for layer in model.model.layers]
    ctrl = opt.qk_clip
    stream = torch.cuda.current_stream(device)

    def probe():
        for module, (q, k) in zip(attn, acts):
            ctrl.record_qk(module, q, k, hd ** -0.5, True, None)
        return ctrl.apply()

    for _ in range(2):
        stats = probe()
    reps = 3
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(reps):
        stats = probe()
    end.record(stream)
    torch.cuda.synchronize()
    probe_ms = start.elapsed_time(end) / reps
    if dist is not None:
        t = torch.tensor([probe_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        probe_ms = float(t.item())
    probe_flops = 2.0 * hq * seq * (seq + 1) / 2.0 * hd * layers   # causal Q K^T

    if rank == 0:
        peaks = load_peaks()
        line = {
            "metric": "MuZO step() ms and QK-Clip probe ms, Llama-3-70B shapes",
            "value": round(dev_ms, 3), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_ms, 3), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init bf16 weights of the named shapes, synthetic SPSA losses, synthetic Q/K)",
            "config": {"workload": "llama3-70b-selected-matrices+qk-probe", "layers": layers,
                       "matrices": len(engine.blocks), "elements": layers * sum(r * c for r, c in SHAPES_70B.values()),
                       "horizon": HORIZON, "ns_steps": 5, "distribution": "normal", "noise_cache": False,
                       "parallelism": f"replica perturb + NS partition x{world}",
                       "probe": f"{layers} layers x B=1 S={seq} Hq={hq} Hkv={hkv} d={hd}, causal"},
            "phase_ms": {k: round(v, 3) for k, v in phases.items()},
            "other_ms": round(dev_ms - sum(phases.values()), 3),
            "ns_tflops": round(ns_tflops, 1), "ns_executed_tflops": round(ns_exec_tflops, 1),
            "ns_frac_of_sustained": round(ns_tflops / peaks["bf16_tflops_sustained"], 4),
            "probe_ms": round(probe_ms, 3),
            "probe_tflops": round(probe_flops / (probe_ms * 1e-3) / 1e12, 1),
            "probe_clip_count": int(stats.qk_clip_count), "probe_smax_max": round(float(stats.qk_smax_max), 3),
            "e2e": {"value": round(run["wall_ms"], 3), "unit": "ms/step"},
            "gpu_launches": int(run["launches"]), "clocks": run["clocks"],
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_reference(args) -> int:
    """The reference's CPU implementation of the path on the host cores: every timed step is one
    matrix of one shape class (the classes in turn, so K steps cover all four when K >= 4), and the
    reported step time is the 224-matrix step extrapolated by count from each class's median.
    Warm-up steps run the smallest class."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cb = _cpu_baseline_module()
    threads = cb.use_all_threads()
    for w in range(args.warmup):
        cb.matrix_step(0, 1000 + w)
    ncls = len(cb.CLASSES)
    samples: dict[int, list[float]] = {c: [] for c in range(ncls)}
    for i in range(max(args.steps, ncls)):
        c = i % ncls
        samples[c].append(sum(cb.matrix_step(c, i)))
    v = cb.step_ms({c: statistics.median(t) for c, t in samples.items()})
    sample = cb.describe(samples, threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 1), "unit": "ms/step", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v, 1), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "horizon": HORIZON, "ns_steps": 5,
                   "distribution": "normal"},
        "cpu_baseline": {"value": round(v, 1), "unit": "ms/step", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 1), "unit": "ms/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- single-kernel cases
# Small, self-contained workloads of one kernel family, used for ncu captures and for the
# Newton-Schulz (batch of 8 per shape) and bandwidth (1 M - 2 G elements, horizon 1-16) sweeps.


L2_FLUSH_BYTES = 512 << 20   # written between timed iterations whose working set could stay in L2


def _event_ms(fn, reps: int, stream, flush: torch.Tensor | None = None) -> float:
    """Mean device time of fn over reps; with `flush`, the buffer is rewritten before each
    iteration (outside the timed interval) so that every iteration starts from a cold L2."""
    if flush is None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in ev:
        flush.add_(1)
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev) / reps


SWEEPS = {
    # Newton-Schulz, batch of 8 per shape (rows x cols)
    "ns": [(1024, 1024), (4096, 4096), (4096, 14336), (14336, 4096), (8192, 28672)],
    # perturbation pass over flat bf16 tensors [numel / 4096, 4096]
    "perturb": [1 << 20, 16 << 20, 256 << 20, 1 << 30, 2 << 30],
    # momentum rebuild horizons
    "rebuild": [1, 2, 4, 8, 16],
}


def _cpu_ns_baseline(rows: int, cols: int, batch: int) -> dict:
    """The reference's CPU Newton-Schulz (fp32) for one matrix of the shape, scaled to the batch;
    the 8192 x 28672 shape (about 3 minutes per matrix on 16 cores) is extrapolated by FLOPs from
    4096 x 14336, the same aspect ratio."""
    from muzo_clip_b200._engine import ns_flops

    cb = _cpu_baseline_module()
    threads = cb.use_all_threads()
    cb.ns_seconds(256, 256)                                                    # warm-up
    if rows * cols > 4096 * 14336:
        r0, c0 = (4096, 14336) if cols >= rows else (14336, 4096)
        sec = cb.ns_seconds(r0, c0) * ns_flops(rows, cols, 5) / ns_flops(r0, c0, 5)
        sample = f"one {r0}x{c0} matrix timed, extrapolated by FLOPs to {rows}x{cols}, x{batch}"
    else:
        sec = cb.ns_seconds(rows, cols)
        sample = f"one {rows}x{cols} matrix timed, x{batch}"
    return {"value": round(sec * batch * 1e3, 1), "unit": "ms per batch", "cores": threads, "kind": "port",
            "dense_tflops": round(batch * ns_flops(rows, cols, 5) / (sec * batch) / 1e12, 3),
            "sample": f"the reference's Newton-Schulz (CPU branch, fp32) on CPU tensors: {sample}"}


def _config1_model(device):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(1234)
    cfg = LlamaConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=4,
                      intermediate_size=688, vocab_size=1024, attn_implementation="eager", initializer_range=0.02)
    return LlamaForCausalLM(cfg).float().to(device)


def _config1_run(opt_cls, device, sync) -> tuple[float, float, int]:
    """Configuration 1 through the public API: the tiny Llama (2 layers, hidden 256, 4 heads, MLP
    688, vocab 1024, fp32), batch 4 x 64 token ids, default hyperparameters, normal noise, 20 SPSA
    steps and one QK-Clip probe. Returns (seconds for the 20 steps, seconds for the probe, steps
    not skipped)."""
    model = _config1_model(device)
    ids = torch.randint(0, 1024, (4, 64), generator=torch.Generator().manual_seed(0)).to(device)
    opt = opt_cls(model, enable_qk_clip=True, seed=1234)

    def closure():
        with torch.no_grad():
            return model(input_ids=ids, labels=ids).loss

    sync()
    t0 = time.perf_counter()
    done = 0
    for _ in range(20):
        opt.estimate_projection(closure)
        done += 0 if opt.step()["skipped"] else 1
    sync()
    t1 = time.perf_counter()
    opt.probe_and_apply_qk_clip(closure, force_eager=True)
    sync()
    t2 = time.perf_counter()
    return t1 - t0, t2 - t1, done


def _run_config1(device) -> dict:
    """This build on the GPU and the reference package itself (``baseline/_ref``, or
    MUZO_REFERENCE_PATH) on the host cores, both through the reference's public API."""
    from muzo_clip_b200 import MuZOClipOptimizer

    sync = torch.cuda.synchronize
    _config1_run(MuZOClipOptimizer, device, sync)                    # warm-up (kernels, transformers)
    gpu_s, gpu_probe_s, gpu_done = _config1_run(MuZOClipOptimizer, device, sync)
    res = {"workload": "tiny Llama (config 1): 20 SPSA steps + one QK-Clip probe, fp32",
           "ms_per_step": round(gpu_s * 1e3 / 20, 3), "probe_ms": round(gpu_probe_s * 1e3, 3),
           "steps_applied": gpu_done}
    ref_root = Path(os.environ.get("MUZO_REFERENCE_PATH", ROOT / "baseline" / "_ref"))
    try:
        if not (ref_root / "muzo_clip").is_dir():
            raise ImportError(f"no reference package under {ref_root}")
        sys.path.insert(0, str(ref_root))
        from muzo_clip import MuZOClipOptimizer as RefOptimizer

        threads = _cpu_baseline_module().use_all_threads()
        cpu = torch.device("cpu")
        ref_s, ref_probe_s, ref_done = _config1_run(RefOptimizer, cpu, lambda: None)
        res["cpu_baseline"] = {"value": round(ref_s * 1e3 / 20, 3), "unit": "ms per step", "cores": threads,
                               "kind": "reference", "probe_ms": round(ref_probe_s * 1e3, 3),
                               "steps_applied": ref_done,
                               "sample": "the reference package itself on CPU tensors (fp32), the same 20 steps "
                                         "and probe"}
    except ImportError as e:
        res["cpu_baseline"] = {"unavailable": str(e)}
    return res


def run_case(args) -> int:
    if not args.sweep:
        return _run_one_case(args)
    for v in SWEEPS[args.case] if args.case in SWEEPS else [None]:
        a = argparse.Namespace(**vars(args))
        if args.case == "ns":
            a.rows, a.cols, a.batch = v[0], v[1], 8
        elif args.case == "perturb":
            a.numel = v
        elif args.case == "rebuild":
            a.horizon = v
        _run_one_case(a)
        torch.cuda.empty_cache()
    return 0


def _run_one_case(args) -> int:
    from muzo_clip_b200 import _lib
    from muzo_clip_b200._engine import ns_flops
    from muzo_clip_b200.newton_schulz import allocate_ns_buffers, ns_iterations

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)
    sp = stream.cuda_stream
    peaks = load_peaks()
    out = {"case": args.case}
    if args.case == "ns":
        buf = allocate_ns_buffers(args.rows, args.cols, args.batch, device)
        buf.x.normal_(0.0, 1.0 / math.sqrt(args.rows * args.cols))
        status = torch.zeros(4, dtype=torch.int32, device=device)
        run = lambda: ns_iterations(buf, args.batch, 5, 0, status.data_ptr(), sp, 0 if args.dense else 1)  # noqa: E731
        for _ in range(args.warmup):
            run()
        ms = _event_ms(run, args.steps, stream)
        fl = args.batch * ns_flops(args.rows, args.cols, 5)
        out.update(rows=args.rows, cols=args.cols, batch=args.batch, symmetric=not args.dense, ms=round(ms, 3),
                   dense_tflops=round(fl / ms / 1e9, 1), status=int(status[0]))
        if args.sweep and not args.no_cpu_baseline:
            out["cpu_baseline"] = _cpu_ns_baseline(args.rows, args.cols, args.batch)
    elif args.case in ("perturb", "rebuild", "apply", "normalize"):
        numel = args.numel
        cols = 4096 if numel % 4096 == 0 else 1
        w = torch.empty((numel // cols, cols), dtype=torch.bfloat16, device=device)
        w.normal_(0.0, 0.02)
        dist_code = _lib.dist_code(args.dist)
        sms, thr = _lib.device_geometry(device)
        keys = torch.tensor(np.arange(1, args.horizon + 1, dtype=np.int64) * 7919, device=device)
        if args.case == "perturb" and args.keep:
            # a later pass of a kept seed: W <- bf16(W + alpha * Zk), Zk written once by a keeping
            # pass (normal noise); W read + written and Zk read: 6 B per element
            zk = torch.empty_like(w)
            segs, total = _lib.plan_segments([numel], [w.data_ptr()], [zk.data_ptr()], _lib.NORMAL, sms, thr)
            table = _lib.to_device_table(segs, device)
            _lib.launch("muzo_perturb_segments_keep_noise", table.data_ptr(), len(segs), total, keys.data_ptr(),
                        _lib.BF16, 1e-3, sp)
            lsegs, ltotal = _lib.plan_linear([numel], [w.data_ptr()], [zk.data_ptr()])
            ltable = _lib.to_device_table(lsegs, device)
            run = lambda: _lib.launch("muzo_perturb_kept_noise", ltable.data_ptr(), len(lsegs), ltotal,  # noqa: E731
                                      _lib.BF16, 1e-3, sp)
            nbytes = 6.0 * numel
        elif args.case == "perturb":
            segs, total = _lib.plan_segments([numel], [w.data_ptr()], None, dist_code, sms, thr)
            table = _lib.to_device_table(segs, device)
            run = lambda: _lib.launch("muzo_perturb_segments", table.data_ptr(), len(segs), total,  # noqa: E731
                                      keys.data_ptr(), _lib.BF16, dist_code, 1e-3, sp)
            nbytes = 4.0 * numel
        elif args.case == "rebuild" and args.keep:
            # every history entry read from a kept-noise slot: H bf16 reads + W read + bf16(M)
            # write = 2H + 4 B per element
            x = torch.empty_like(w)
            pool = torch.empty((args.horizon, numel), dtype=torch.bfloat16, device=device)
            pool.normal_()
            lsegs, ltotal = _lib.plan_linear([numel], [w.data_ptr()], [x.data_ptr()])
            lsegs["kept"] = [0]
            table = _lib.to_device_table(lsegs, device)
            bases = torch.tensor([pool[h].data_ptr() for h in range(args.horizon)], dtype=torch.int64, device=device)
            alphas = torch.full((args.horizon,), 0.1, dtype=torch.float32, device=device)
            sums = torch.zeros(_lib.NSUMS, dtype=torch.float64, device=device)
            flags = torch.zeros(4, dtype=torch.int32, device=device)
            run = lambda: _lib.launch("muzo_rebuild_kept_linear", table.data_ptr(), len(lsegs), ltotal,  # noqa: E731
                                      alphas.data_ptr(), bases.data_ptr(), args.horizon, _lib.BF16, 1, 0.5,
                                      sums.data_ptr(), flags.data_ptr(), sp)
            nbytes = (2.0 * args.horizon + 4.0) * numel
        elif args.case == "rebuild":
            x = torch.empty_like(w)
            segs, total = _lib.plan_segments([numel], [w.data_ptr()], [x.data_ptr()], dist_code, sms, thr)
            table = _lib.to_device_table(segs, device)
            alphas = torch.full((args.horizon,), 0.1, dtype=torch.float32, device=device)
            sums = torch.zeros(_lib.NSUMS, dtype=torch.float64, device=device)
            flags = torch.zeros(4, dtype=torch.int32, device=device)
            run = lambda: _lib.launch("muzo_rebuild_segments", table.data_ptr(), len(segs), total,  # noqa: E731
                                      keys.data_ptr(), alphas.data_ptr(), args.horizon, dist_code, _lib.BF16, 1, 0.5,
                                      sums.data_ptr(), flags.data_ptr(), 0, sp)
            nbytes = 4.0 * numel  # bf16(M) write + W read
        else:
            # the update apply (X read, W read + written: 6 B per element) or the normalisation of
            # the rebuilt momentum (X read + written: 4 B per element), on one block
            x = torch.empty_like(w)
            x.normal_(0.0, 1.0 / math.sqrt(numel))
            segs, total = _lib.plan_linear([numel], [w.data_ptr()], [x.data_ptr()])
            table = _lib.to_device_table(segs, device)
            sums = torch.zeros(_lib.NSUMS, dtype=torch.float64, device=device)
            sums[_lib.SUM_X2] = 1.0
            sums[_lib.SUM_M2] = 1.0
            sums[_lib.SUM_W2] = numel * 0.02 ** 2
            sums[_lib.SUM_U2] = float(numel)
            flags = torch.zeros(4, dtype=torch.int32, device=device)
            stats = torch.zeros(_lib.NSTATS, dtype=torch.float32, device=device)
            scales = torch.ones(1, dtype=torch.float32, device=device)
            if args.case == "apply":
                run = lambda: _lib.launch("muzo_apply_update", table.data_ptr(), len(segs), total,  # noqa: E731
                                          _lib.BF16, scales.data_ptr(), 1e-5, 0.01, 1, 1.0 - 1e-7, sums.data_ptr(),
                                          flags.data_ptr(), stats.data_ptr(), sp)
                nbytes = 6.0 * numel
            else:
                run = lambda: _lib.launch("muzo_ns_normalize", table.data_ptr(), len(segs), total,  # noqa: E731
                                          sums.data_ptr(), flags.data_ptr(), sp)
                nbytes = 4.0 * numel
        for _ in range(args.warmup):
            run()
        # working sets below 1 GiB (8 x the 126 MB L2) could be partly served from L2 on repeated
        # passes: flush between them
        flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device) if nbytes < 2 * L2_FLUSH_BYTES \
            else None
        ms = _event_ms(run, args.steps, stream, flush)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out.update(numel=numel, dist="kept" if args.keep and args.case in ("perturb", "rebuild") else args.dist,
                   horizon=args.horizon if args.case == "rebuild" else None,
                   ms=round(ms, 4), gbs=round(gbs, 1), hbm_frac=round(gbs / peaks["hbm_gbs"], 4),
                   l2="flushed between passes" if flush is not None else "working set larger than L2")
        if args.case == "perturb" and args.sweep and not args.keep and not args.no_cpu_baseline \
                and numel <= (256 << 20):
            cb = _cpu_baseline_module()
            threads = cb.use_all_threads()
            cb.perturb_pass_seconds(min(numel, 1 << 20), args.dist)          # warm-up
            cpu_s = statistics.median(cb.perturb_pass_seconds(numel, args.dist, i) for i in range(3))
            out["cpu_baseline"] = {"value": round(cpu_s * 1e3, 3), "unit": "ms per pass", "cores": threads,
                                   "kind": "port", "gbs": round(4.0 * numel / cpu_s / 1e9, 2),
                                   "sample": f"the reference's perturbation op sequence on CPU tensors ({args.dist} "
                                             f"noise from the CPU generator), median of 3 passes"}
    elif args.case == "config1":
        out.update(_run_config1(device))
    elif args.case == "attn":
        # one attention layer with the per-head max-logit side output (the fused capture path)
        # against SDPA plus the separate max-logit kernel on the same states
        from muzo_clip_b200 import _qk

        b, hq, hkv, seq, d = args.batch, args.heads, args.kv_heads, args.seq, args.head_dim
        q = torch.randn((b, seq, hq, d), device=device, dtype=torch.bfloat16).transpose(1, 2)
        k = torch.randn((b, seq, hkv, d), device=device, dtype=torch.bfloat16).transpose(1, 2)
        v = torch.randn((b, seq, hkv, d), device=device, dtype=torch.bfloat16).transpose(1, 2)
        fused = lambda: _qk.attention_max(q, k, v, d ** -0.5, True)  # noqa: E731

        def separate():
            torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=d ** -0.5,
                                                             enable_gqa=True)
            _qk.qk_head_max(q, k, d ** -0.5, True, None)

        sdpa = lambda: torch.nn.functional.scaled_dot_product_attention(  # noqa: E731
            q, k, v, is_causal=True, scale=d ** -0.5, enable_gqa=True)
        res = {}
        for name, fn in (("fused", fused), ("sdpa_plus_max", separate), ("sdpa", sdpa)):
            for _ in range(args.warmup):
                fn()
            res[name] = _event_ms(fn, args.steps, stream)
        flops = 4.0 * b * hq * seq * seq * d / 2.0  # Q K^T and P V, causal half
        out.update(batch=b, heads=hq, kv_heads=hkv, seq=seq, head_dim=d,
                   ms_fused=round(res["fused"], 4), ms_sdpa_plus_max=round(res["sdpa_plus_max"], 4),
                   ms_sdpa=round(res["sdpa"], 4), fused_tflops=round(flops / res["fused"] / 1e9, 1),
                   sdpa_tflops=round(flops / res["sdpa"] / 1e9, 1))
    elif args.case == "qk":
        # per-head max logit of one attention layer: Q [B, Hq, S, D], K [B, Hkv, S, D] as the
        # transposed views of [B, S, H, D] that transformers passes to attention functions
        from muzo_clip_b200 import _qk

        b, hq, hkv, seq, d = args.batch, args.heads, args.kv_heads, args.seq, args.head_dim
        q = torch.randn((b, seq, hq, d), device=device, dtype=torch.bfloat16).transpose(1, 2)
        k = torch.randn((b, seq, hkv, d), device=device, dtype=torch.bfloat16).transpose(1, 2)
        run = lambda: _qk.qk_head_max(q, k, d ** -0.5, True, None)  # noqa: E731
        for _ in range(args.warmup):
            run()
        ms = _event_ms(run, args.steps, stream)
        flops = 2.0 * b * hq * seq * seq * d / 2.0  # causal half
        out.update(batch=b, heads=hq, kv_heads=hkv, seq=seq, head_dim=d, ms_per_layer=round(ms, 4),
                   causal_tflops=round(flops / ms / 1e9, 1))
    else:
        raise SystemExit(f"unknown case {args.case}")
    print(json.dumps(out), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None,
                    choices=["ns", "perturb", "rebuild", "apply", "normalize", "qk", "attn", "config1"],
                    help="run one kernel family on a small workload instead of the optimizer step")
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--cols", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--dense", action="store_true", help="ns case: compute every output tile")
    ap.add_argument("--numel", type=int, default=1 << 28)
    ap.add_argument("--dist", default="rademacher", choices=["normal", "rademacher"])
    ap.add_argument("--horizon", type=int, default=8)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=64)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="muzo", choices=["muzo", "reference"])
    ap.add_argument("--layers", type=int, default=None, help="layers (default 32, or 80 for llama3-70b)")
    ap.add_argument("--workload", default="llama3-8b", choices=["llama3-8b", "llama3-70b"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--keep", action="store_true",
                    help="perturb case: a pass that reads kept noise (muzo_perturb_kept_noise); rebuild case: "
                         "every history entry read from kept noise (muzo_rebuild_kept_linear)")
    ap.add_argument("--no-noise-cache", action="store_true",
                    help="time only the default configuration (every pass and history entry regenerates its noise)")
    ap.add_argument("--no-variant", action="store_true",
                    help="skip the regenerated-noise variant timed before the kept-noise line")
    ap.add_argument("--sweep", action="store_true",
                    help="with --case: ns = 5 shapes x batch 8; perturb = 1 M..2 G elements; rebuild = horizon 1..16")
    args = ap.parse_args()
    if args.case is not None:
        return run_case(args)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "llama3-70b":
        return run_70b(args)
    if args.layers is None:
        args.layers = LAYERS
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
