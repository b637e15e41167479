"""Host logic of the sharded step on two gloo ranks (CPU, no GPU).

Covers: the LPT ownership is identical on every rank; owners' updated blocks reach every rank
through the broadcasts of the collective exchange; per-block statistics scattered into global
buffers and summed over the group give every rank every block's statistics; the peer exchange's
address table; the SPSA losses are averaged over the group so every rank derives the same
projection; QK-Clip maxima captured on per-rank batches are max-reduced so every rank clips alike.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


class _Block:
    def __init__(self, index, rows, cols, tensor):
        self.index, self.rows, self.cols, self.tensor, self.dtype = index, rows, cols, tensor, tensor.dtype
        self.numel = rows * cols


def _worker(rank: int, world: int, store: str, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT / "muzo-clip_b200"))
    # file rendezvous: no TCP port to race for on a shared host
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world)
    try:
        import numpy as np

        from muzo_clip_b200 import _lib
        from muzo_clip_b200._engine import StepEngine, ns_flops, partition_blocks
        from muzo_clip_b200.distributed import ShardedStepEngine

        shapes = [(64, 32), (16, 32), (16, 32), (64, 32), (96, 32), (96, 32), (32, 96)] * 3
        blocks = [_Block(i, r, c, torch.full((r, c), -1.0)) for i, (r, c) in enumerate(shapes)]
        owner = partition_blocks([ns_flops(r, c, 5) for r, c in shapes], world)

        class Fake:  # the host and collective parts of ShardedStepEngine on CPU tensors
            _after_class = ShardedStepEngine._after_class
            _finish_collectives = ShardedStepEngine._finish_collectives
            _class_blocks = ShardedStepEngine._class_blocks
            _broadcast = ShardedStepEngine._broadcast
            scatter_owned_results = ShardedStepEngine.scatter_owned_results
            reduce_results = ShardedStepEngine.reduce_results
            _read_results = ShardedStepEngine._read_results
            _stats_from = StepEngine._stats_from
            gather_stats = ShardedStepEngine.gather_stats
            _code = staticmethod(ShardedStepEngine._code)

        eng = Fake()
        eng.blocks, eng.owner, eng.world, eng.group = blocks, owner, world, dist.group.WORLD
        eng._pending, eng._handles, eng._global_ranks, eng.device = [], [], list(range(world)), torch.device("cpu")
        eng.exchange, eng._peer = "nccl", None
        owned = [b for b in blocks if owner[b.index] == rank]
        # the step's per-block state of this rank's blocks, in slot order, as _build_step lays it out
        n_owned, n = len(owned), len(blocks)
        eng.n_slots = n_owned
        eng.sums_bytes = 8 * _lib.NSUMS * max(n_owned, 1)
        eng.flags_off = eng.sums_bytes
        eng.stats_off = (eng.flags_off + 4 * (max(n_owned, 1) + 4) + 15) // 16 * 16
        eng.state_bytes = eng.stats_off + 4 * _lib.NSTATS * max(n_owned, 1)
        eng.state = torch.zeros(eng.state_bytes, dtype=torch.uint8)
        sums = eng.state[:eng.sums_bytes].view(torch.float64).view(-1, _lib.NSUMS)
        flags = eng.state[eng.flags_off:eng.flags_off + 4 * (max(n_owned, 1) + 4)].view(torch.int32)
        stats = eng.state[eng.stats_off:eng.state_bytes].view(torch.float32).view(-1, _lib.NSTATS)
        for slot, b in enumerate(owned):
            numel = b.rows * b.cols
            sums[slot, _lib.SUM_W2] = numel * 0.02 ** 2          # rms(W) = 0.02
            sums[slot, _lib.SUM_U2_CLIPPED] = numel * (1.0 + b.index) ** 2   # rms(U) = 1 + index
            stats[slot, _lib.STAT_CLIP_FACTOR] = 0.5
            flags[slot] = b.index % 2
        ShardedStepEngine._alloc_global_results(eng, n)
        eng.owned_global = torch.tensor([b.index for b in owned], dtype=torch.int64)
        # owners "update" their blocks; everyone else holds stale values
        for b in owned:
            b.tensor.fill_(float(b.index))
        class_order = []
        for b in blocks:
            ck = (b.rows, b.cols, eng._code(b))
            if ck not in class_order:
                class_order.append(ck)
        for ck in class_order:
            eng._after_class(ck)
        eng._finish_collectives()
        ok = all(bool((b.tensor == float(b.index)).all()) for b in blocks)
        lr = 1e-3
        per_block = eng.gather_stats(eng._read_results(lr))
        want_rms = {b.index: float(np.float32(np.float32(1.0 + b.index) * np.float32(lr))) for b in blocks}
        stats_ok = sorted(per_block) == list(range(n)) and all(
            abs(per_block[i]["update_rms"] - want_rms[i]) <= 1e-6 * want_rms[i] and per_block[i]["clip"] == 0.5
            and per_block[i]["flags"] == i % 2 for i in per_block)

        # loss averaging of estimate_projection over the group
        import muzo_clip_b200.muzo_optimizer as mo

        class FakeEngine:
            def __init__(self, opt, *a, **k):
                self.device = torch.device("cpu")

            def matches(self, opt):
                return True

            def perturb(self, seed, alpha):
                pass

        mo.StepEngine = FakeEngine
        mo.MuZOClipOptimizer._engine_for_step = lambda self: self._engine or setattr(self, "_engine", FakeEngine(self)) or self._engine
        model = torch.nn.Module()
        model.q_proj = torch.nn.Linear(8, 8, bias=False)
        opt = mo.MuZOClipOptimizer(model, seed=3, process_group=dist.group.WORLD)
        losses = iter([1.0 + rank, 1.5 + 2 * rank])
        proj = opt.estimate_projection(lambda: next(losses))
        t = torch.tensor([proj["p_raw"], proj["seed"] % 1000003], dtype=torch.float64)
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        same_p = all(torch.equal(g, gathered[0]) for g in gathered)
        Path(out_dir, f"rank{rank}.txt").write_text(f"{int(ok)} {int(stats_ok)} {int(same_p)} {owner}\n")
    finally:
        dist.destroy_process_group()


def test_sharded_collectives_on_two_gloo_ranks(tmp_path):
    """NCCL-style exchange (broadcasts) and the global per-block statistics, summed over the
    group: every rank ends with every block's final value and every block's statistics."""
    world = 2
    mp.start_processes(_worker, args=(world, str(tmp_path / "store"), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    lines = [Path(tmp_path, f"rank{r}.txt").read_text().split(" ", 3) for r in range(world)]
    for ok, stats_ok, same_p, owner in lines:
        assert ok == "1" and stats_ok == "1" and same_p == "1"
    assert lines[0][3] == lines[1][3]  # identical ownership on both ranks


def test_peer_destinations_open_each_handle_once():
    """The peer exchange's address table from the handles every rank exported: one mapping per
    distinct (rank, allocation), every owned block's address in every peer = base + offset."""
    sys.path.insert(0, str(ROOT / "muzo-clip_b200"))
    from muzo_clip_b200.distributed import peer_destinations

    world, nblocks = 3, 5
    # rank r's blocks 0-2 share one allocation, blocks 3-4 another
    gathered = [[(b"h%d-%d" % (r, 0 if i < 3 else 1), 4096 * i) for i in range(nblocks)] for r in range(world)]
    opened = []

    def opener(handle):
        opened.append(handle)
        return 1 << 40 | (len(opened) << 32)

    dst, bases = peer_destinations(gathered, [0, 3, 4], 1, opener)
    assert sorted(dst) == [0, 2] and len(opened) == len(set(opened)) == 4
    for r in (0, 2):
        assert sorted(dst[r]) == [0, 3, 4]
        for i in (0, 3, 4):
            handle, off = gathered[r][i]
            assert dst[r][i] == bases[(r, handle)] + off


def _qk_worker(rank: int, world: int, store: str, out_dir: str) -> None:
    from datetime import timedelta

    sys.path.insert(0, str(ROOT / "muzo-clip_b200"))
    # a short timeout: a rank left waiting in a collective fails the test instead of hanging it
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    try:
        from muzo_clip_b200.qk_clip import QKClipController

        model = torch.nn.Module()
        model.layers = torch.nn.ModuleList()
        for _ in range(3):
            attn = torch.nn.Module()
            attn.q_proj = torch.nn.Linear(8, 8, bias=False)
            attn.k_proj = torch.nn.Linear(8, 4, bias=False)
            model.layers.append(attn)
        ctl = QKClipController(model, tau=1.0, process_group=dist.group.WORLD)
        inf = float("inf")
        # rank 0 saw layers 0 and 2, rank 1 saw layers 0 and 1 (e.g. a capture dropped for
        # non-finite logits); -inf is a head with no visible logit
        mine = {0: {"layers.0": [1.0, 5.0, 2.0, 3.0], "layers.2": [0.5, -inf]},
                1: {"layers.0": [4.0, 0.0, 2.0, -inf], "layers.1": [7.0, 8.0, 9.0]}}[rank]
        for name, vals in mine.items():
            ctl._captured_smax[name] = torch.tensor(vals, dtype=torch.float32)
        ctl.reduce_over_group()
        got = {n: t.tolist() for n, t in ctl._captured_smax.items()}
        want = {"layers.0": [4.0, 5.0, 2.0, 3.0], "layers.1": [7.0, 8.0, 9.0], "layers.2": [0.5, -inf]}
        # nothing captured anywhere: stays empty on every rank
        ctl.clear()
        ctl.reduce_over_group()
        empty = not ctl._captured_smax
        # head counts that differ between the ranks: every rank raises, none is left waiting
        ctl._captured_smax["layers.1"] = torch.zeros(4 if rank == 0 else 3)
        try:
            ctl.reduce_over_group()
            raised = False
        except ValueError:
            raised = True
        dist.barrier()   # the group still works afterwards
        Path(out_dir, f"qk{rank}.txt").write_text(f"{int(got == want)} {int(empty)} {int(raised)}\n")
    finally:
        dist.destroy_process_group()


def test_qk_clip_maxima_reduced_over_two_gloo_ranks(tmp_path):
    world = 2
    mp.start_processes(_qk_worker, args=(world, str(tmp_path / "store"), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    for r in range(world):
        assert Path(tmp_path, f"qk{r}.txt").read_text().split() == ["1", "1", "1"], r


def test_collective_order_is_global_for_any_ownership():
    """Each rank calls the class collectives in the global class order even when it owns no
    block of some classes (the loop of StepEngine.run_step)."""
    sys.path.insert(0, str(ROOT / "muzo-clip_b200"))
    from muzo_clip_b200._engine import StepEngine

    src = Path(StepEngine.run_step.__code__.co_filename).read_text()
    assert "while next_class < len(self.class_order)" in src


def _stall_worker(rank: int, world: int, store: str, out_dir: str) -> None:
    import time
    from datetime import timedelta

    sys.path.insert(0, str(ROOT / "muzo-clip_b200"))
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=4))
    try:
        if rank == 1:
            time.sleep(12)   # never joins the projection's loss all-reduce
            return
        import muzo_clip_b200.muzo_optimizer as mo

        class FakeEngine:
            def __init__(self, opt, *a, **k):
                self.device = torch.device("cpu")

            def matches(self, opt):
                return True

            def perturb(self, seed, alpha):
                pass

        mo.MuZOClipOptimizer._engine_for_step = lambda self: self._engine or setattr(self, "_engine", FakeEngine(self)) or self._engine
        model = torch.nn.Module()
        model.q_proj = torch.nn.Linear(8, 8, bias=False)
        opt = mo.MuZOClipOptimizer(model, seed=3, process_group=dist.group.WORLD)
        t0 = time.monotonic()
        try:
            opt.estimate_projection(lambda: 1.0)
            outcome = "returned"
        except Exception as exc:  # the collective's timeout error of the backend
            outcome = type(exc).__name__
        waited = time.monotonic() - t0
        Path(out_dir, "stall.txt").write_text(f"{outcome} {waited:.1f} {len(opt.history)}\n")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_stalled_rank_ends_the_others_collective_with_an_error(tmp_path):
    """A rank that stops answering (here: never joins the SPSA loss all-reduce that ends a
    projection) makes the other rank's collective fail within the process group's timeout
    (4 s) instead of waiting for ever; the projection then raises and appends nothing to the
    history (muzo_optimizer.py:213-215 re-raises exceptions of a projection)."""
    world = 2
    mp.start_processes(_stall_worker, args=(world, str(tmp_path / "store"), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    outcome, waited, hist = Path(tmp_path, "stall.txt").read_text().split()
    assert outcome != "returned" and float(waited) < 11.0 and hist == "0", (outcome, waited, hist)
