"""Generate the CUDA golden vectors of the reference path with torch on a B200.

Runs the reference's tensor-op sequence (oracle/torch_reference.py, itself proven equal to the reference
package by check_against_reference.py) on a CUDA device and stores small fixtures:
  noise_cuda.npz    torch CUDA generator output for several sizes (full arrays for small tensors,
                    fixed index samples for large ones, including tensors torch splits into
                    several launches)
  step_cuda.npz     perturbation, momentum rebuild, Newton-Schulz and update results
  meta.json         device name, torch version, SM count and threads per SM
Usage: python tests/golden/gen_cuda_golden.py --out tests/golden
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1] / "oracle"))

import torch_reference as tr  # noqa: E402

# (name, numel, distribution, storage): "full" keeps every value, "sample" keeps fixed indices
NOISE_CASES = [
    ("n1", 1, "normal", "full"),
    ("n7", 7, "normal", "full"),
    ("n1000", 1000, "normal", "full"),
    ("n65539", 65539, "normal", "full"),
    ("n1212433", 303104 * 4 + 17, "normal", "sample"),
    ("n4194304", 1 << 22, "normal", "sample"),
    ("n_split", (1 << 29) + 1000, "normal", "sample"),
    ("r1", 1, "rademacher", "full"),
    ("r1000", 1000, "rademacher", "full"),
    ("r65539", 65539, "rademacher", "full"),
    ("r1212433", 303104 * 4 + 17, "rademacher", "full"),
    ("r4194304", 1 << 22, "rademacher", "sample"),
    ("r_split", (1 << 31) + 64, "rademacher", "sample"),
]


def sample_indices(numel: int, threads: int, extra_boundaries=()) -> np.ndarray:
    rng = np.random.default_rng(numel)
    pts = set(range(min(64, numel)))
    pts.update(range(max(0, numel - 64), numel))
    for b in list(extra_boundaries) + [threads * k for k in range(1, 9)]:
        for d in range(-8, 8):
            if 0 <= b + d < numel:
                pts.add(b + d)
    pts.update(rng.integers(0, numel, size=min(4096, numel)).tolist())
    return np.asarray(sorted(pts), dtype=np.int64)


def noise_key(name: str) -> int:
    return tr.hash64_seed(20260101, f"golden.{name}.weight", (1, 1), 0)


@torch.no_grad()
def gen_noise(device) -> dict:
    out = {}
    props = torch.cuda.get_device_properties(device)
    threads = min(1184, props.multi_processor_count * props.max_threads_per_multi_processor // 256) * 256
    for name, numel, dist, storage in NOISE_CASES:
        key = noise_key(name)
        gen = torch.Generator(device=device)
        gen.manual_seed(key)
        if dist == "normal":
            z = torch.randn((numel,), generator=gen, device=device, dtype=torch.float32)
        else:
            z = torch.randint(0, 2, (numel,), generator=gen, device=device, dtype=torch.int8)
        out[f"{name}.key"] = np.asarray([key], dtype=np.uint64)
        out[f"{name}.numel"] = np.asarray([numel], dtype=np.int64)
        if storage == "full":
            idx = np.arange(numel, dtype=np.int64)
        else:
            idx = sample_indices(numel, threads, extra_boundaries=(numel // 2, numel // 4, 3 * numel // 4))
        vals = z[torch.from_numpy(idx).to(device)].cpu().numpy()
        if dist == "rademacher" and storage == "full":
            out[f"{name}.bits"] = np.packbits(vals.astype(np.uint8))
        else:
            out[f"{name}.idx"] = idx
            out[f"{name}.val"] = vals.astype(np.float32 if dist == "normal" else np.int8)
        del z
        torch.cuda.empty_cache()
    return out


class _Item:
    def __init__(self, seed, p):
        self.seed, self.p = seed, p


@torch.no_grad()
def gen_step(device) -> dict:
    out = {}
    g = torch.Generator().manual_seed(1234)
    hist = [_Item(int(torch.randint(0, 2**62, (1,), generator=g)), float(torch.randn((), generator=g).clamp(-3, 3)))
            for _ in range(5)]
    out["hist.seed"] = np.asarray([h.seed for h in hist], dtype=np.uint64)
    out["hist.p"] = np.asarray([h.p for h in hist], dtype=np.float64)
    for dist in ("normal", "rademacher"):
        for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            w0 = (torch.randn((64, 128), generator=g) * 0.02).to(dt)
            w = w0.to(device)
            tr.perturb([("golden.perturb.weight", w)], 77, 1.0, 1e-3, dist)
            out[f"perturb.{dist}.{dt_name}.in"] = w0.float().numpy()
            out[f"perturb.{dist}.{dt_name}.out"] = w.float().cpu().numpy()
            blk = w0.to(device)
            M = tr.rebuild(blk, "golden.rebuild.weight", 0, hist, 0.9, dist, True)
            out[f"rebuild.{dist}.{dt_name}.M"] = M.cpu().numpy()
    for shape in ((64, 96), (96, 64), (256, 688), (688, 256)):
        G = torch.randn(shape, generator=g)
        X = tr.newton_schulz(G.to(device), 5)
        out[f"ns.{shape[0]}x{shape[1]}.G"] = G.numpy()
        out[f"ns.{shape[0]}x{shape[1]}.X"] = X.cpu().numpy()
    # update on a bf16 block with the Newton-Schulz result as U (clipped and unclipped)
    for tag, lr in (("clip", 1e-2), ("noclip", 1e-6)):
        w0 = (torch.randn((96, 64), generator=g) * 0.02).to(torch.bfloat16)
        G = torch.randn((96, 64), generator=g)
        U = tr.newton_schulz(G.to(device), 5)
        blk = w0.to(device)
        urms, ratio = tr.apply_update(blk, U.clone(), lr, 0.2, 0.01, 0.01)
        out[f"apply.{tag}.w0"] = w0.float().numpy()
        out[f"apply.{tag}.U"] = U.cpu().numpy()
        out[f"apply.{tag}.w1"] = blk.float().cpu().numpy()
        out[f"apply.{tag}.stats"] = np.asarray([urms, ratio, lr], dtype=np.float64)
    # QK logits maxima (eager path) with GQA and causal masking
    for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        q = torch.randn((2, 4, 48, 32), generator=g).to(dt)
        k = torch.randn((2, 2, 48, 32), generator=g).to(dt)
        logits = tr.eager_logits(q.to(device), k.to(device), 32 ** -0.5, True)
        out[f"qk.{dt_name}.q"] = q.float().numpy()
        out[f"qk.{dt_name}.k"] = k.float().numpy()
        out[f"qk.{dt_name}.smax"] = tr.qk_head_max(logits).numpy()
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--skip-large", action="store_true")
    args = ap.parse_args()
    if not torch.cuda.is_available():
        print("a CUDA device is required", file=sys.stderr)
        return 2
    device = torch.device("cuda", 0)
    if args.skip_large:
        NOISE_CASES[:] = [c for c in NOISE_CASES if "split" not in c[0]]
    outdir = Path(args.out)
    outdir.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(outdir / "noise_cuda.npz", **gen_noise(device))
    np.savez_compressed(outdir / "step_cuda.npz", **gen_step(device))
    props = torch.cuda.get_device_properties(device)
    meta = {"device": props.name, "torch": torch.__version__, "sm_count": props.multi_processor_count,
            "max_threads_per_sm": props.max_threads_per_multi_processor}
    (outdir / "meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("wrote", outdir)
    return 0


if __name__ == "__main__":
    sys.exit(main())
