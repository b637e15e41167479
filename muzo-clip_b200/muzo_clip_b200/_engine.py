"""Device-side engine of MuZOClipOptimizer: launch tables, key uploads and the step pipeline.

Everything model-sized stays on the GPU. Per perturbation pass the host computes one 63-bit key
per parameter block (cached per seed), uploads them, and one kernel launch per parameter dtype
regenerates the noise and updates every block in place. Per step the owned blocks are processed
in batches of equal shape: rebuild -> normalise -> Newton-Schulz GEMMs (the last one also sums
the update's squares) -> apply, and the step statistics come back in one device-to-host copy.
"""

from __future__ import annotations

import logging
import math
import os
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np
import torch

from . import _lib
from .newton_schulz import NSBuffers, ns_buffers_in, ns_iterations, ns_workspace_bytes
from .prng import hash64_seed, iter_param_blocks

DEFAULT_WORKSPACE_BYTES = 16 << 30

logger = logging.getLogger(__name__)


@dataclass
class Block:
    index: int              # position in the optimizer's block list
    name: str
    block_index: int
    tensor: torch.Tensor    # view into param.data
    rows: int
    cols: int
    dtype: torch.dtype

    @property
    def numel(self) -> int:
        return self.rows * self.cols

    def key(self, seed: int) -> int:
        return hash64_seed(seed, self.name, (self.rows, self.cols), self.block_index)


@dataclass
class PerturbGroup:
    dtype_code: int
    blocks: list[Block]
    table: torch.Tensor
    nsegs: int
    total_items: int
    # kept noise, per slot of the noise pool: the first pass of a seed stores dtype(Z) (keep:
    # noise segments whose out is the block's place in the slot), later passes of that seed read
    # it back (kept: linear segments, param = block, out = its noise); (table, nsegs, items)
    keep_tables: dict[int, tuple[torch.Tensor, int, int]] = field(default_factory=dict)
    kept_tables: dict[int, tuple[torch.Tensor, int, int]] = field(default_factory=dict)


@dataclass
class Chunk:
    blocks: list[Block]
    rows: int
    cols: int
    dtype_code: int
    slot0: int                   # first index of this chunk in the step's per-block arrays
    rebuild_table: torch.Tensor
    rebuild_nsegs: int
    rebuild_items: int
    norm_table: torch.Tensor
    norm_items: int
    # every history entry kept: linear segments (param = block, out = bf16(M), kept = the block's
    # byte offset in a noise slot)
    kept_rebuild_table: torch.Tensor | None = None
    kept_rebuild_items: int = 0
    apply_tables: dict[int, tuple[torch.Tensor, int]] = field(default_factory=dict)  # by parity
    scales: torch.Tensor | None = None
    pad_views: list[torch.Tensor] | None = None
    buf: NSBuffers | None = None


class _Uploader:
    """Ring of pinned host staging buffers for small per-step uploads (keys, coefficients)."""

    def __init__(self, device: torch.device, nbytes: int, depth: int = 4):
        self.device = device
        self.nbytes = max(int(nbytes), 64)
        self.host = [torch.empty(self.nbytes, dtype=torch.uint8, pin_memory=True) for _ in range(depth)]
        self.dev = [torch.empty(self.nbytes, dtype=torch.uint8, device=device) for _ in range(depth)]
        self.events = [None] * depth
        self.i = 0

    def upload(self, arr: np.ndarray) -> torch.Tensor:
        raw = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
        if raw.size > self.nbytes:
            raise ValueError("upload larger than the staging buffer")
        i = self.i
        self.i = (i + 1) % len(self.host)
        if self.events[i] is not None:
            self.events[i].synchronize()
        h = self.host[i]
        h[: raw.size].numpy()[:] = raw
        d = self.dev[i]
        d[: raw.size].copy_(h[: raw.size], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.events[i] = ev
        return d


def ns_flops(rows: int, cols: int, steps: int) -> float:
    """Dense FLOPs of the quintic iteration on one rows x cols matrix: 5 * (4 m^2 n + 2 m^3)."""
    m, n = min(rows, cols), max(rows, cols)
    return float(steps) * (4.0 * m * m * n + 2.0 * m ** 3)


def partition_blocks(costs: Sequence[float], world: int) -> list[int]:
    """Owner rank of every block: longest-processing-time greedy over the given costs
    (ties resolved by block index, so every rank computes the same assignment)."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0.0] * world
    owner = [0] * len(costs)
    for i in order:
        r = min(range(world), key=lambda q: (load[q], q))
        owner[i] = r
        load[r] += costs[i]
    return owner


class StepEngine:
    def __init__(self, opt, rank: int = 0, world: int = 1, process_group=None):
        self.opt = opt
        self.rank = rank
        self.world = world
        self.pg = process_group
        blocks: list[Block] = []
        for sel in opt.selected_params:
            data = sel.param.data
            if data.device.type != "cuda":
                raise ValueError(f"muzo_clip_b200 needs CUDA parameters; {sel.name} is on {data.device}")
            for bi, _, view in iter_param_blocks(data, opt.block_rows):
                if not view.is_contiguous():
                    raise ValueError(f"parameter block {sel.name}[{bi}] is not contiguous")
                _lib.dtype_code(view.dtype)
                blocks.append(Block(len(blocks), sel.name, bi, view, int(view.shape[0]), int(view.shape[1]),
                                    view.dtype))
        self.blocks = blocks
        self.device = blocks[0].tensor.device if blocks else torch.device("cuda")
        self.fingerprint = self._fingerprint(opt)
        self.dist = _lib.dist_code(opt.distribution)
        self.sms, self.max_thr = _lib.device_geometry(self.device)
        self._key_cache: dict[int, np.ndarray] = {}
        # kept noise (normal noise only: Rademacher passes are close to the HBM rate already): a
        # pool of slots, each holding one projection's rounded noise for every block, so that the
        # later passes of a projection and the rebuild of every history entry that still has a
        # slot read the noise instead of regenerating it
        self.keep_noise = bool(getattr(opt, "noise_cache", False)) and self.dist == _lib.NORMAL
        self.noise_pool: torch.Tensor | None = None
        self.slot_bytes = 0
        self.slot_seed: list[int | None] = []
        self._noise_offsets: list[int] = []
        self.kept_entries = 0     # history entries the last rebuild read from kept noise
        self._build_perturb_groups()
        costs = [ns_flops(b.rows, b.cols, max(opt.ns_steps, 1)) for b in blocks]
        self.owner = partition_blocks(costs, world) if world > 1 else [0] * len(blocks)
        self.owned = [b for b in blocks if self.owner[b.index] == rank]
        self._step_ready = False
        self._phase_events = None
        # optional observer of every batch's Newton-Schulz result, called as
        # hook(blocks, x, stream) with x the [batch, rows, cols] bf16 result in the matrices' own
        # layout, after the GEMMs and before the update is applied (parity tests read it there)
        self.ns_output_hook = None
        # nonzero: written to the Newton-Schulz GEMMs' stall-request word (status word 3) for the
        # next steps, making that role's bounded wait expire (tests of the timeout path)
        self.gemm_stall_request = 0
        # rebuild of batch i+1 on a side stream (one CTA per SM) while batch i is on the tensor
        # cores; off by default: the GEMMs already run at the power cap
        self.overlap = os.environ.get("MUZO_OVERLAP_REBUILD", "0") == "1"
        horizon = max(opt.horizon, 1)
        self.uploader = _Uploader(self.device, 8 * (len(blocks) * (horizon + 1) + 2 * horizon + 64))

    # ------------------------------------------------------------------ bookkeeping
    @staticmethod
    def _fingerprint(opt) -> tuple:
        return tuple((s.name, s.param.data.data_ptr(), tuple(s.param.shape), s.param.dtype)
                     for s in opt.selected_params) + (opt.block_rows, opt.distribution,
                                                      bool(getattr(opt, "noise_cache", False)))

    def matches(self, opt) -> bool:
        return self.fingerprint == self._fingerprint(opt)

    def keys_for(self, seed: int) -> np.ndarray:
        keys = self._key_cache.get(seed)
        if keys is None:
            keys = np.fromiter((b.key(seed) for b in self.blocks), dtype=np.uint64, count=len(self.blocks))
            if len(self._key_cache) > self.opt.horizon + 4:
                self._key_cache.pop(next(iter(self._key_cache)))
            self._key_cache[seed] = keys
        return keys

    # ------------------------------------------------------------------ perturbation
    def _build_perturb_groups(self) -> None:
        groups: dict[int, list[Block]] = {}
        for b in self.blocks:
            groups.setdefault(_lib.dtype_code(b.dtype), []).append(b)
        self.perturb_groups: list[PerturbGroup] = []
        for code, blks in groups.items():
            segs, total = _lib.plan_segments([b.numel for b in blks], [b.tensor.data_ptr() for b in blks],
                                             None, self.dist, self.sms, self.max_thr)
            # block_index in the table indexes the group's key array
            table = _lib.to_device_table(segs, self.device)
            self.perturb_groups.append(PerturbGroup(code, blks, table, len(segs), total))
        if self.keep_noise:
            self._build_noise_buffer()

    NOISE_POOL_RESERVE = 24 << 30   # device memory left free for the workspace and the rest

    def _build_noise_buffer(self) -> None:
        """The noise pool: up to horizon + 1 slots (the projection being evaluated and every
        history entry), each one buffer of the rounded noise of every block in the block's dtype
        and layout (256-byte aligned places), as many as fit next to 24 GiB left free (at most
        MUZO_NOISE_SLOTS). Left out, with a warning, when not even one slot fits."""
        offsets, total = [], 0
        for b in self.blocks:
            offsets.append(total)
            total += (b.numel * b.tensor.element_size() + 255) // 256 * 256
        total = max(total, 256)
        free, _ = torch.cuda.mem_get_info(self.device)
        want = max(int(self.opt.horizon), 1) + 1
        cap = os.environ.get("MUZO_NOISE_SLOTS")
        if cap:
            want = min(want, max(int(cap), 0))
        fit = max(0, (free - self.NOISE_POOL_RESERVE) // total)
        if fit == 0 and total <= free // 2:   # small devices: one slot, at most half the free memory
            fit = 1
        nslots = int(min(want, fit))
        if nslots < 1:
            logger.warning("noise_cache needs %.1f GB of device memory per projection, more than is free (%.1f GB); "
                           "every pass regenerates its noise instead", total / 1e9, free / 1e9)
            self.keep_noise = False
            return
        self.noise_pool = torch.empty(nslots * total, dtype=torch.uint8, device=self.device)
        self.slot_bytes = total
        self.slot_seed = [None] * nslots
        self._noise_offsets = offsets

    def slot_base(self, slot: int) -> int:
        return self.noise_pool.data_ptr() + slot * self.slot_bytes

    def _slot_tables(self, g: PerturbGroup, slot: int):
        """(keep, kept) tables of a perturbation group for one slot, built on first use."""
        if slot not in g.keep_tables:
            base = self.slot_base(slot)
            numels = [b.numel for b in g.blocks]
            params = [b.tensor.data_ptr() for b in g.blocks]
            outs = [base + self._noise_offsets[b.index] for b in g.blocks]
            segs, items = _lib.plan_segments(numels, params, outs, self.dist, self.sms, self.max_thr)
            g.keep_tables[slot] = (_lib.to_device_table(segs, self.device), len(segs), items)
            lsegs, litems = _lib.plan_linear(numels, params, outs)
            g.kept_tables[slot] = (_lib.to_device_table(lsegs, self.device), len(lsegs), litems)
        return g.keep_tables[slot], g.kept_tables[slot]

    def slot_of(self, seed: int) -> int | None:
        """Slot holding the complete noise of `seed`, if any."""
        for i, sd in enumerate(self.slot_seed):
            if sd == seed:
                return i
        return None

    def _free_slot(self) -> int:
        """A slot for a new projection's noise: an empty one, else one whose seed left the
        history, else the one holding the oldest history entry (that entry is then regenerated
        until it leaves the history)."""
        live = [item.seed for item in self.opt.history]
        for i, sd in enumerate(self.slot_seed):
            if sd is None:
                return i
        for i, sd in enumerate(self.slot_seed):
            if sd not in live:
                return i
        oldest = {sd: age for age, sd in enumerate(live)}
        return min(range(len(self.slot_seed)), key=lambda i: oldest.get(self.slot_seed[i], -1))

    def perturb(self, seed: int, alpha: float) -> None:
        """W <- W + alpha * Z(seed) for every selected block (muzo_optimizer.py:434-446). With the
        noise pool, the first pass of a seed also keeps dtype(Z) in a slot and every later pass of
        the same seed reads it back: the same values without regenerating the noise."""
        if not self.blocks:
            return
        stream = _lib.stream_ptr(self.device)
        alpha32 = float(np.float32(alpha))
        slot = self.slot_of(seed) if self.keep_noise else None
        if slot is not None:
            self._mark("perturb", True)
            for g in self.perturb_groups:
                _, (table, nsegs, items) = self._slot_tables(g, slot)
                _lib.launch("muzo_perturb_kept_noise", table.data_ptr(), nsegs, items, g.dtype_code, alpha32, stream)
            self._mark("perturb", False)
            return
        keys = self.keys_for(seed)
        dev_keys = self.uploader.upload(keys)
        if self.keep_noise:
            slot = self._free_slot()
            self.slot_seed[slot] = None  # being rewritten
        self._mark("perturb", True)
        for g in self.perturb_groups:
            idx = np.fromiter((b.index for b in g.blocks), dtype=np.int64, count=len(g.blocks))
            if len(self.perturb_groups) == 1 and np.array_equal(idx, np.arange(len(self.blocks))):
                kptr = dev_keys.data_ptr()
            else:
                kptr = self.uploader.upload(keys[idx]).data_ptr()
            if slot is not None:
                (table, nsegs, items), _ = self._slot_tables(g, slot)
                _lib.launch("muzo_perturb_segments_keep_noise", table.data_ptr(), nsegs, items, kptr, g.dtype_code,
                            alpha32, stream)
            else:
                _lib.launch("muzo_perturb_segments", g.table.data_ptr(), g.nsegs, g.total_items, kptr,
                            g.dtype_code, self.dist, alpha32, stream)
        self._mark("perturb", False)
        if slot is not None:
            self.slot_seed[slot] = seed

    # ------------------------------------------------------------------ step
    def _workspace_budget(self) -> int:
        budget = getattr(self.opt, "workspace_bytes", None) or DEFAULT_WORKSPACE_BYTES
        try:
            free, _ = torch.cuda.mem_get_info(self.device)
            budget = min(budget, int(free * 0.5))
        except RuntimeError:
            pass
        return max(budget, 1)

    def _build_step(self) -> None:
        """Plan the step: shape classes in a global order (cheapest rebuild first, identical on
        every rank), batches of owned blocks per class sized to half the workspace budget, and
        two workspace slots used alternately so that the rebuild of batch i+1 (side stream) can
        run while batch i is on the tensor cores."""
        opt = self.opt
        first_seen: dict[tuple[int, int, int], int] = {}
        for b in self.blocks:
            first_seen.setdefault((b.rows, b.cols, _lib.dtype_code(b.dtype)), len(first_seen))
        desc = self._descending_classes()
        self.class_order = sorted(first_seen, key=lambda ck: ((-1 if desc else 1) * ck[0] * ck[1], first_seen[ck]))
        owned_by_class: dict[tuple[int, int, int], list[Block]] = {ck: [] for ck in self.class_order}
        for b in self.owned:
            owned_by_class[(b.rows, b.cols, _lib.dtype_code(b.dtype))].append(b)
        slot_budget = max(self._workspace_budget() // 2, 1)
        plans = []
        for ck in self.class_order:
            blks = owned_by_class[ck]
            if not blks:
                continue
            rows, cols, _ = ck
            per_block = ns_workspace_bytes(rows, cols, 1)
            cap = max(1, min(len(blks), slot_budget // per_block))
            nchunks = -(-len(blks) // cap)
            size = -(-len(blks) // nchunks)
            for start in range(0, len(blks), size):
                plans.append((ck, blks[start:start + size]))
        slot_bytes = max((ns_workspace_bytes(ck[0], ck[1], len(part)) for ck, part in plans), default=256)
        nslots = 2 if len(plans) > 1 else 1
        self.slots = [torch.empty(slot_bytes, dtype=torch.uint8, device=self.device) for _ in range(nslots)]
        self.chunks: list[Chunk] = []
        stat_slot = 0
        for i, ((rows, cols, code), part) in enumerate(plans):
            n = len(part)
            buf = ns_buffers_in(self.slots[i % nslots], rows, cols, n)
            dense = buf.ld == cols
            # rebuild and normalise write X0 densely; padded layouts go through a staging copy
            if dense:
                x0_ptrs = [buf.x_slot(0)[j].data_ptr() for j in range(n)]
                pad_views = None
            else:
                stage = torch.empty((n, rows, cols), dtype=torch.bfloat16, device=self.device)
                x0_ptrs = [stage[j].data_ptr() for j in range(n)]
                pad_views = [stage]
            rsegs, rtot = _lib.plan_segments([b.numel for b in part], [b.tensor.data_ptr() for b in part],
                                             x0_ptrs, self.dist, self.sms, self.max_thr)
            if self.keep_noise:
                # kept history entries are read at slot base + the block's offset in a slot
                rsegs["kept"] = [self._noise_offsets[part[int(bi)].index] for bi in rsegs["block_index"]]
            nsegs, ntot = _lib.plan_linear([b.numel for b in part], x0_ptrs, x0_ptrs)
            ch = Chunk(part, rows, cols, code, stat_slot, _lib.to_device_table(rsegs, self.device), len(rsegs), rtot,
                       _lib.to_device_table(nsegs, self.device), ntot, pad_views=pad_views)
            if self.keep_noise:
                ksegs, ktot = _lib.plan_linear([b.numel for b in part], [b.tensor.data_ptr() for b in part], x0_ptrs)
                ksegs["kept"] = [self._noise_offsets[b.index] for b in part]
                ch.kept_rebuild_table, ch.kept_rebuild_items = _lib.to_device_table(ksegs, self.device), ktot
            ch.buf = buf
            for parity in (0, 1):
                xs = buf.x_slot(parity)
                outs = [xs[j].data_ptr() for j in range(n)] if dense else x0_ptrs
                asegs, atot = _lib.plan_linear([b.numel for b in part], [b.tensor.data_ptr() for b in part], outs)
                ch.apply_tables[parity] = (_lib.to_device_table(asegs, self.device), atot)
            scales = np.asarray([math.sqrt(max(b.rows, b.cols)) * opt.muon_scale for b in part], dtype=np.float32)
            ch.scales = torch.from_numpy(scales).to(self.device)
            self.chunks.append(ch)
            stat_slot += n
        self.n_slots = stat_slot
        self.side_stream = torch.cuda.Stream(self.device)
        # one zeroed device buffer per step: sums (f64), flags + status (i32), stats (f32)
        self.sums_bytes = 8 * _lib.NSUMS * max(stat_slot, 1)
        self.flags_off = self.sums_bytes
        self.stats_off = self.flags_off + 4 * (max(stat_slot, 1) + 4)
        self.stats_off = (self.stats_off + 15) // 16 * 16
        self.state_bytes = self.stats_off + 4 * _lib.NSTATS * max(stat_slot, 1)
        self.state = torch.zeros(self.state_bytes, dtype=torch.uint8, device=self.device)
        self._step_ready = True

    def owned_ns_flops(self) -> float:
        return sum(ns_flops(b.rows, b.cols, self.opt.ns_steps) for b in self.owned)

    def owned_ns_flops_executed(self) -> float:
        """FLOPs the tensor cores execute: X X^T and b A + c A A only on the tiles that meet the
        upper triangle (256 x 256 CTA-pair tiles for m >= 256, else 128 x 256 one-SM tiles),
        a X + B X in full."""
        tot = 0.0
        for b in self.owned:
            m, n = min(b.rows, b.cols), max(b.rows, b.cols)
            bm = 256 if m >= 256 else 128
            tm, tn = -(-m // bm), -(-m // 256)
            frac = sum(tn - (r * bm) // 256 for r in range(tm)) / float(tm * tn)
            tot += self.opt.ns_steps * (frac * (2.0 * m * m * n + 2.0 * m ** 3) + 2.0 * m * m * n)
        return tot

    def start_phase_timing(self) -> None:
        self._phase_events = {}

    def stop_phase_timing(self) -> dict[str, float]:
        """Milliseconds per phase accumulated since start_phase_timing (synchronises)."""
        ev_map, self._phase_events = self._phase_events or {}, None
        torch.cuda.synchronize(self.device)
        return {k: sum(a.elapsed_time(b) for a, b in v) for k, v in ev_map.items()}

    def profile_step(self, history, lr: float) -> dict[str, float]:
        """Run one step with CUDA events around each phase; returns milliseconds per phase
        (summed over chunks). Applies the update like run_step."""
        self._phase_events: dict[str, list] = {}
        try:
            self.run_step(history, lr)
            torch.cuda.synchronize(self.device)
            return {k: sum(a.elapsed_time(b) for a, b in v) for k, v in self._phase_events.items()}
        finally:
            self._phase_events = None

    def _mark(self, phase: str, start: bool, stream=None) -> None:
        """Phase boundary: an NVTX range (muzo/<phase>) for profilers and, while phase timing is
        on, a CUDA event on the phase's stream."""
        if start:
            torch.cuda.nvtx.range_push(f"muzo/{phase}")
        else:
            torch.cuda.nvtx.range_pop()
        ev_map = getattr(self, "_phase_events", None)
        if ev_map is None:
            return
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream if stream is not None else torch.cuda.current_stream(self.device))
        if start:
            ev_map.setdefault(phase, []).append([ev, None])
        else:
            ev_map[phase][-1][1] = ev

    def run_step(self, history, lr: float) -> dict[int, dict[str, float]]:
        """Rebuild, orthogonalise and apply the update of every owned block. Returns per-block
        statistics keyed by block index (owned blocks only)."""
        opt = self.opt
        if not self._step_ready:
            self._build_step()
        hist = list(reversed(history))
        horizon = len(hist)
        coeffs = [opt.beta_momentum ** age for age in range(horizon)]
        coeff_sum = 0.0
        for c in coeffs:
            coeff_sum += c
        alphas = np.asarray([c * item.p for c, item in zip(coeffs, hist)], dtype=np.float32)
        normalize = 1 if (opt.normalize_momentum and coeff_sum > 0) else 0
        inv_cs = float(np.float32(1.0) / np.float32(coeff_sum)) if normalize else 1.0
        stream = _lib.stream_ptr(self.device)
        device = self.device

        # keys of every owned block for every history item, chunk-major: [slot, age]
        seed_keys = [self.keys_for(item.seed) for item in hist]
        order = np.fromiter((b.index for ch in self.chunks for b in ch.blocks), dtype=np.int64,
                            count=self.n_slots)
        keys = np.stack([k[order] for k in seed_keys], axis=1) if horizon else np.zeros((0, 0), np.uint64)
        # the slot of every history entry whose noise is kept (0: regenerate)
        slots = [self.slot_of(item.seed) if self.keep_noise else None for item in hist]
        slot_base = np.asarray([0 if sl is None else self.slot_base(sl) for sl in slots], dtype=np.uint64)
        self.kept_entries = sum(sl is not None for sl in slots)
        payload = np.concatenate([slot_base.view(np.uint8), keys.reshape(-1).view(np.uint8), alphas.view(np.uint8)])
        dev = self.uploader.upload(payload)
        slot_base_ptr = dev.data_ptr()
        keys_ptr = slot_base_ptr + 8 * horizon
        alphas_ptr = keys_ptr + keys.size * 8
        self._slot_base_ptr = slot_base_ptr
        self.state.zero_()
        base = self.state.data_ptr()
        sums_ptr, flags_ptr, stats_ptr = base, base + self.flags_off, base + self.stats_off
        status_ptr = flags_ptr + 4 * (max(self.n_slots, 1))
        if self.gemm_stall_request:
            self.state.view(torch.int32)[(status_ptr - base) // 4 + 3] = int(self.gemm_stall_request)
        lr32 = float(np.float32(lr))
        decay = float(np.float32(1.0 - lr * opt.weight_decay))
        apply_decay = 1 if opt.weight_decay else 0
        compute = torch.cuda.current_stream(self.device)
        side = self.side_stream if self.overlap else compute
        inputs_ready = torch.cuda.Event()
        inputs_ready.record(compute)
        side.wait_event(inputs_ready)
        done: list[torch.cuda.Event] = []
        args = (horizon, keys_ptr, alphas_ptr, normalize, inv_cs, sums_ptr, flags_ptr, stats_ptr, status_ptr, lr32,
                decay, apply_decay)
        next_class = 0
        for i, ch in enumerate(self.chunks):
            # rebuild + normalise on the side stream once the slot's previous user has finished
            if i >= 2:
                side.wait_event(done[i - 2])
            self._prepare_chunk(ch, side, *args)
            ready = torch.cuda.Event()
            ready.record(side)
            compute.wait_event(ready)
            self._finish_chunk(ch, compute, *args)
            self._after_chunk(ch, compute)
            ev = torch.cuda.Event()
            ev.record(compute)
            done.append(ev)
            ck = (ch.rows, ch.cols, ch.dtype_code)
            last_of_class = i + 1 == len(self.chunks) or (self.chunks[i + 1].rows, self.chunks[i + 1].cols,
                                                          self.chunks[i + 1].dtype_code) != ck
            if last_of_class:
                # collectives run class by class in the global order on every rank, including
                # classes this rank owns nothing of
                while next_class < len(self.class_order):
                    cur = self.class_order[next_class]
                    next_class += 1
                    self._after_class(cur)
                    if cur == ck:
                        break
        while next_class < len(self.class_order):
            self._after_class(self.class_order[next_class])
            next_class += 1
        self._finish_collectives()
        return self._read_results(lr32)

    def _prepare_chunk(self, ch, stream, horizon, keys_ptr, alphas_ptr, normalize, inv_cs, sums_ptr, flags_ptr,
                       stats_ptr, status_ptr, lr32, decay, apply_decay) -> None:
        sp = stream.cuda_stream
        n = len(ch.blocks)
        s_sums = sums_ptr + 8 * _lib.NSUMS * ch.slot0
        s_flags = flags_ptr + 4 * ch.slot0
        self._mark("rebuild", True, stream)
        max_ctas = self.sms if self.overlap else 0
        if self.kept_entries and self.kept_entries == horizon:
            _lib.launch("muzo_rebuild_kept_linear", ch.kept_rebuild_table.data_ptr(), n, ch.kept_rebuild_items,
                        alphas_ptr, self._slot_base_ptr, horizon, ch.dtype_code, normalize, inv_cs, s_sums, s_flags,
                        sp)
        elif self.kept_entries:
            _lib.launch("muzo_rebuild_segments_history", ch.rebuild_table.data_ptr(), ch.rebuild_nsegs,
                        ch.rebuild_items, keys_ptr + 8 * horizon * ch.slot0, alphas_ptr, self._slot_base_ptr,
                        horizon, ch.dtype_code, normalize, inv_cs, s_sums, s_flags, max_ctas, sp)
        else:
            _lib.launch("muzo_rebuild_segments", ch.rebuild_table.data_ptr(), ch.rebuild_nsegs, ch.rebuild_items,
                        keys_ptr + 8 * horizon * ch.slot0, alphas_ptr, horizon, self.dist, ch.dtype_code,
                        normalize, inv_cs, s_sums, s_flags, max_ctas, sp)
        self._mark("rebuild", False, stream)
        self._mark("normalize", True, stream)
        _lib.launch("muzo_ns_normalize", ch.norm_table.data_ptr(), n, ch.norm_items, s_sums, s_flags, sp)
        self._mark("normalize", False, stream)
        if ch.pad_views is not None:
            with torch.cuda.stream(stream):
                ch.buf.x_slot(0)[:n, :, : ch.cols].copy_(ch.pad_views[0])

    def _finish_chunk(self, ch, stream, horizon, keys_ptr, alphas_ptr, normalize, inv_cs, sums_ptr, flags_ptr,
                      stats_ptr, status_ptr, lr32, decay, apply_decay) -> None:
        opt = self.opt
        sp = stream.cuda_stream
        n = len(ch.blocks)
        s_sums = sums_ptr + 8 * _lib.NSUMS * ch.slot0
        s_flags = flags_ptr + 4 * ch.slot0
        s_stats = stats_ptr + 4 * _lib.NSTATS * ch.slot0
        self._mark("ns", True, stream)
        # the last GEMM also sums U^2 per block and flags a non-finite result
        parity = ns_iterations(ch.buf, n, opt.ns_steps, 0, status_ptr, sp, sums_ptr=s_sums,
                               scales_ptr=ch.scales.data_ptr(), flags_ptr=s_flags)
        self._mark("ns", False, stream)
        if ch.pad_views is not None:
            with torch.cuda.stream(stream):
                ch.pad_views[0].copy_(ch.buf.x_slot(parity)[:n, :, : ch.cols])
        if self.ns_output_hook is not None:
            x = ch.pad_views[0] if ch.pad_views is not None else ch.buf.x_slot(parity)[:n]
            self.ns_output_hook(ch.blocks, x, stream)
        table, items = ch.apply_tables[parity if ch.pad_views is None else 0]
        self._mark("apply", True, stream)
        if opt.ns_steps <= 0:  # no GEMM: the normalised momentum itself is the update
            _lib.launch("muzo_update_sumsq", table.data_ptr(), n, items, ch.scales.data_ptr(), s_sums, s_flags, sp)
        _lib.launch("muzo_apply_update", table.data_ptr(), n, items, ch.dtype_code, ch.scales.data_ptr(), lr32,
                    float(opt.update_ratio_clip), apply_decay, decay, s_sums, s_flags, s_stats, sp)
        self._mark("apply", False, stream)

    # hooks for the sharded (multi-GPU) engine
    def _descending_classes(self) -> bool:
        """Shape classes largest first (per-class collectives) instead of smallest first."""
        return os.environ.get("MUZO_COLLECTIVES", "end") == "class"

    def _after_chunk(self, ch, stream) -> None:
        """The blocks of `ch` are final once the work queued on `stream` so far has run."""

    def _after_class(self, class_key) -> None:
        pass

    def _finish_collectives(self) -> None:
        pass

    def _read_results(self, lr32: float) -> dict[int, dict[str, float]]:
        """The step's per-block results in one device-to-host copy (owned blocks only)."""
        host = self.state.cpu().numpy()
        n = max(self.n_slots, 1)
        sums = host[: self.sums_bytes].view(np.float64).reshape(n, _lib.NSUMS)
        flags = host[self.flags_off: self.flags_off + 4 * (n + 4)].view(np.int32)
        stats = host[self.stats_off: self.stats_off + 4 * _lib.NSTATS * n].view(np.float32).reshape(n, _lib.NSTATS)
        pairs, slot = [], 0
        for ch in self.chunks:
            for b in ch.blocks:
                pairs.append((b, slot))
                slot += 1
        return self._stats_from(sums, flags, stats, int(flags[n]), pairs, lr32)

    def _stats_from(self, sums, flags, stats, status: int, pairs, lr32: float) -> dict[int, dict[str, float]]:
        """Per-block statistics (muzo_optimizer.py:342-357) from the step's sums, flags and
        statistics; `pairs` lists (block, row of that block in the arrays)."""
        if status != 0:
            raise _lib.MuzoError(f"Newton-Schulz GEMM reported status {status} (a bounded wait expired); the "
                                 "weights this step updated are unspecified: restore them from a checkpoint")
        out: dict[int, dict[str, float]] = {}
        lr = np.float32(lr32)
        for b, slot in pairs:
            s = sums[slot]
            st = stats[slot]
            numel = float(b.numel)
            zeroed = bool(st[_lib.STAT_ZEROED] != 0)
            rms_w = np.float32(math.sqrt(s[_lib.SUM_W2] / numel))
            denom = np.float32(rms_w + np.float32(1e-12))
            if zeroed:
                update_rms, ratio = 0.0, 0.0
            else:
                rms_u = np.float32(math.sqrt(s[_lib.SUM_U2_CLIPPED] / numel))
                update_rms_f = np.float32(rms_u * lr)
                update_rms = float(update_rms_f)
                ratio = float(np.float32(update_rms_f / denom))
            out[b.index] = {
                "update_rms": update_rms,
                "ratio": ratio,
                "ratio_before": float(st[_lib.STAT_RATIO_BEFORE]),
                "clip": float(st[_lib.STAT_CLIP_FACTOR]),
                "zeroed": zeroed,
                "flags": int(flags[slot]),
            }
        return out
