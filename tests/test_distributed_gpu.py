"""The sharded step on 2 GPUs (NCCL, one process per GPU) against one GPU.

Every rank perturbs its own replica; each block is rebuilt, orthogonalised and applied by its
owner only and placed in the other rank's replica (copy-engine pushes through peer mappings, or
NCCL broadcasts). With the same seeds and losses the weights must come out
bit-identical on both ranks and equal to the single-GPU run: the kernels work per matrix, so the
partition and the batch composition change nothing. With per-rank batches (each rank's closure
returns its own loss) the ranks average the two SPSA losses, so they must match one GPU whose
closure returns that mean. QK-Clip maxima captured on per-rank batches are max-reduced before
the clip: both ranks' q/k weights must equal one GPU clipping with the element-wise maximum.
Skipped with fewer than 2 GPUs.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
SHAPES = [(512, 256), (256, 512), (1024, 256), (384, 384), (256, 768), (768, 256), (512, 256), (256, 256)]
STEPS = 6


def _build(device):
    torch.manual_seed(5)
    model = torch.nn.Module()
    model.layers = torch.nn.ModuleList()
    for rows, cols in SHAPES:
        blk = torch.nn.Module()
        blk.up_proj = torch.nn.Linear(cols, rows, bias=False)
        model.layers.append(blk)
    return model.to(device=device, dtype=torch.bfloat16)


# per-rank batch offsets of the loss; 2-rank sums and halving are exact in fp64, so one GPU can
# reproduce the all-reduced mean bit for bit
RANK_SHIFT = (1.0, -1.0)


def _run(model, process_group=None, shift=None, noise_cache=False) -> dict[str, torch.Tensor]:
    """``shift``: None (same batch everywhere), a rank's own offset, or "mean" (one GPU playing
    both ranks)."""
    from muzo_clip_b200 import MuZOClipOptimizer

    opt = MuZOClipOptimizer(model, seed=21, horizon=4, min_history=2, process_group=process_group,
                            noise_cache=noise_cache)
    w0 = model.layers[0].up_proj.weight

    def closure():
        f = float(w0.float().square().sum().item())
        if shift is None:
            return f
        if shift == "mean":
            return ((f + RANK_SHIFT[0]) + (f + RANK_SHIFT[1])) / 2.0
        return f + shift

    for _ in range(STEPS):
        opt.estimate_projection(closure)
        opt.step()
    torch.cuda.synchronize()
    out = {n: p.detach().cpu() for n, p in model.named_parameters()}
    if hasattr(opt._engine, "close"):
        if process_group is not None:
            import torch.distributed as dist

            dist.barrier(group=process_group)   # no peer still pushes into this rank
        opt._engine.close()
    return out


def _worker(rank: int, world: int, store: str, out_prefix: str, own_batches: bool = False, exchange: str = "peer",
            noise_cache: bool = False) -> None:
    sys.path.insert(0, str(ROOT / "muzo-clip_b200"))
    os.environ.update(NCCL_NVLS_ENABLE="0", MUZO_EXCHANGE=exchange)
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    # file rendezvous: no TCP port to race for on a shared host
    dist.init_process_group("nccl", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        weights = _run(_build(torch.device("cuda", rank)), dist.group.WORLD,
                       RANK_SHIFT[rank] if own_batches else None, noise_cache)
        torch.save(weights, f"{out_prefix}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("own_batches,exchange,noise_cache", [(False, "peer", False), (True, "peer", False),
                                                             (False, "nccl", False), (True, "peer", True)],
                         ids=["same_batch-peer", "per_rank_batches-peer", "same_batch-nccl", "per_rank-peer-kept"])
def test_two_ranks_match_one_gpu(tmp_path, own_batches, exchange, noise_cache):
    """Peer exchange (owners push their blocks into the other rank's parameters with copy-engine
    copies) and NCCL broadcasts; with and without the kept-noise pool."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ref = _run(_build(torch.device("cuda", 0)), shift="mean" if own_batches else None)
    mp.start_processes(_worker, args=(2, str(tmp_path / "store"), str(tmp_path / "w"), own_batches, exchange,
                                      noise_cache), nprocs=2, start_method="spawn", join=True)
    moved = sum(int(not torch.equal(ref[n], v)) for n, v in _build(torch.device("cpu")).named_parameters())
    assert moved == len(SHAPES)  # every selected matrix was updated
    for r in range(2):
        got = torch.load(tmp_path / f"w.{r}")
        for name, value in ref.items():
            assert torch.equal(value, got[name]), (r, name)


QK_MAXIMA = {  # per rank: module -> per-head maxima of its own batch (tau = 10)
    0: {"layers.0": [12.0, 3.0, 30.0, 9.0], "layers.1": [1.0, 2.0, 3.0, 4.0]},
    1: {"layers.0": [11.0, 25.0, 2.0, float("-inf")], "layers.2": [40.0, 5.0, 6.0, 7.0]},
}


def _qk_model(device):
    torch.manual_seed(9)
    model = torch.nn.Module()
    model.layers = torch.nn.ModuleList()
    for _ in range(3):
        attn = torch.nn.Module()
        attn.q_proj = torch.nn.Linear(64, 4 * 16, bias=False)   # 4 heads of 16
        attn.k_proj = torch.nn.Linear(64, 2 * 16, bias=False)   # 2 KV heads (GQA groups of 2)
        model.layers.append(attn)
    return model.to(device=device, dtype=torch.bfloat16)


def _qk_apply(device, maxima, process_group=None):
    from muzo_clip_b200.qk_clip import QKClipController

    model = _qk_model(device)
    ctl = QKClipController(model, tau=10.0, alpha=0.5, process_group=process_group)
    for name, vals in maxima.items():
        ctl._captured_smax[name] = torch.tensor(vals, dtype=torch.float32, device=device)
    stats = ctl.apply()
    torch.cuda.synchronize()
    return {n: p.detach().cpu() for n, p in model.named_parameters()}, stats


def _qk_worker(rank: int, world: int, store: str, out_prefix: str) -> None:
    sys.path.insert(0, str(ROOT / "muzo-clip_b200"))
    os.environ.update(NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        weights, stats = _qk_apply(torch.device("cuda", rank), QK_MAXIMA[rank], dist.group.WORLD)
        torch.save((weights, stats.qk_clip_count, stats.qk_smax_max), f"{out_prefix}.{rank}")
    finally:
        dist.destroy_process_group()


def test_qk_clip_with_per_rank_batches_matches_one_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    merged: dict[str, list[float]] = {}
    for per_rank in QK_MAXIMA.values():
        for name, vals in per_rank.items():
            prev = merged.get(name, [float("-inf")] * len(vals))
            merged[name] = [max(a, b) for a, b in zip(prev, vals)]
    ref, ref_stats = _qk_apply(torch.device("cuda", 0), merged)
    assert ref_stats.qk_clip_count > 0
    mp.start_processes(_qk_worker, args=(2, str(tmp_path / "store"), str(tmp_path / "qk")), nprocs=2,
                       start_method="spawn", join=True)
    for r in range(2):
        weights, count, smax = torch.load(tmp_path / f"qk.{r}")
        assert (count, smax) == (ref_stats.qk_clip_count, ref_stats.qk_smax_max), r
        for name, value in ref.items():
            assert torch.equal(value, weights[name]), (r, name)
