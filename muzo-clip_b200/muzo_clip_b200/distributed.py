"""Sharded step over the ranks of a torch.distributed process group (one process per GPU).

Every rank keeps a full replica of the selected weights. Perturbation needs no communication:
the noise of a block is a pure function of (seed, name, shape, block index), so all ranks
perturb their replicas identically. The step is partitioned: blocks are assigned to ranks by
Newton-Schulz FLOPs (LPT greedy, identical on every rank); each rank rebuilds, orthogonalises and
applies only its blocks and then places them in every other rank's replica.

Weight exchange (``MUZO_EXCHANGE``):

* ``peer`` (default when the parameter memory can be shared between the node's processes): once,
  every rank exports the interprocess handles of the allocations that hold its parameters and
  maps the peers'. After each batch of blocks is applied, the owner pushes those blocks straight
  into every peer's parameters with copy-engine copies (one cudaMemcpyAsync per block, one stream
  per peer), so the transfer runs under the Newton-Schulz GEMMs of the following batches without
  taking their SMs. Batches go largest shape class first, so the last batch, whose transfer is not
  hidden, is the smallest.
* ``nccl``: once the last GEMM is queued, the owners broadcast the updated blocks with NCCL, all
  in one group (also the fallback when a rank cannot share its parameter memory).

Per-block statistics: every rank scatters its blocks' sums, flags and statistics into buffers
indexed by global block and sums them over the group with one all-reduce on the device; the host
reads them with the step's single device-to-host copy. In the ``peer`` exchange that all-reduce
also waits for every rank's pushes, so when it completes on a rank, every block has arrived there:
the rank's stream waits for it before the weights are used again. The pushes start only after the
SPSA loss all-reduce that ends every projection (every rank has finished its perturbation passes).
"""

from __future__ import annotations

import ctypes
import logging
import os

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from ._engine import StepEngine

logger = logging.getLogger(__name__)


def export_handles(blocks) -> list[tuple[bytes, int]] | None:
    """(handle bytes, offset) of the allocation holding every block, or None when one of them
    cannot be shared between processes."""
    out = []
    for b in blocks:
        h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        off = ctypes.c_uint64(0)
        size = ctypes.c_uint64(0)
        st = _lib.lib.muzo_ipc_export(b.tensor.data_ptr(), h, ctypes.byref(off), ctypes.byref(size))
        if st != _lib.OK:
            return None
        out.append((h.raw, int(off.value)))
    return out


def peer_destinations(gathered, owned_indices, rank: int, opener) -> tuple[dict, dict]:
    """Destination address of every owned block in every peer's replica, from the handle lists
    all ranks gathered. `opener(handle)` maps a peer's handle once (each distinct (rank, handle)
    is opened once). Returns ({peer: {block index: address}}, {(peer, handle): mapped base})."""
    bases: dict[tuple[int, bytes], int] = {}
    dst: dict[int, dict[int, int]] = {}
    world = len(gathered)
    for step in range(1, world):
        r = (rank + step) % world
        dst[r] = {}
        for i in owned_indices:
            handle, off = gathered[r][i]
            key = (r, handle)
            if key not in bases:
                bases[key] = opener(handle)
            dst[r][i] = bases[key] + off
    return dst, bases


class PeerExchange:
    """Copy-engine pushes of owned blocks into the peers' parameter memory (IPC mappings)."""

    def __init__(self, engine, gathered):
        self.engine = engine
        self.rank, self.world = engine.rank, engine.world

        def opener(handle: bytes) -> int:
            base = ctypes.c_void_p(0)
            _lib.check(_lib.lib.muzo_ipc_import(handle, ctypes.byref(base)), "muzo_ipc_import")
            return int(base.value)

        self.dst, self.bases = peer_destinations(gathered, [b.index for b in engine.owned], self.rank, opener)
        self.streams = {r: torch.cuda.Stream(engine.device) for r in self.dst}

    def push(self, blocks, ready: torch.cuda.Event) -> None:
        """Queue the copies of `blocks` (final on this rank once `ready` has passed) to every peer."""
        if not blocks:
            return
        torch.cuda.nvtx.range_push("muzo/push")
        src = np.asarray([b.tensor.data_ptr() for b in blocks], dtype=np.uint64)
        nbytes = np.asarray([b.numel * b.tensor.element_size() for b in blocks], dtype=np.uint64)
        for r, stream in self.streams.items():
            stream.wait_event(ready)
            dst = np.asarray([self.dst[r][b.index] for b in blocks], dtype=np.uint64)
            _lib.launch("muzo_push_blocks", dst.ctypes.data, src.ctypes.data, nbytes.ctypes.data, len(blocks),
                        stream.cuda_stream)
        torch.cuda.nvtx.range_pop()

    def join(self, stream: torch.cuda.Stream) -> None:
        """Make `stream` wait for every push queued so far."""
        for s in self.streams.values():
            stream.wait_stream(s)

    def close(self) -> None:
        for base in self.bases.values():
            _lib.lib.muzo_ipc_close(base)
        self.bases = {}


class ShardedStepEngine(StepEngine):
    def __init__(self, opt, process_group):
        self.group = process_group
        rank = dist.get_rank(process_group)
        world = dist.get_world_size(process_group)
        super().__init__(opt, rank=rank, world=world, process_group=process_group)
        self._pending: list = []
        self._handles: list = []
        self._global_ranks = [dist.get_global_rank(process_group, r) if process_group is not None else r
                              for r in range(world)] if process_group is not None else list(range(world))
        want = os.environ.get("MUZO_EXCHANGE", "peer")
        self.exchange = "peer" if (want == "peer" and world > 1 and self.device.type == "cuda") else "nccl"
        self._peer: PeerExchange | None = None

    # ------------------------------------------------------------------ set-up
    def _descending_classes(self) -> bool:
        return self.exchange == "peer" or super()._descending_classes()

    def _build_step(self) -> None:
        super()._build_step()
        self._alloc_global_results(len(self.blocks))
        order = [b.index for ch in self.chunks for b in ch.blocks]
        self.owned_global = torch.tensor(order, dtype=torch.int64, device=self.device)
        self.comm_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        if self.exchange == "peer" and self._peer is None:
            mine = export_handles(self.blocks)
            gathered = [None] * self.world
            dist.all_gather_object(gathered, mine, group=self.group)
            if all(g is not None for g in gathered):
                self._peer = PeerExchange(self, gathered)
            else:
                logger.warning("parameter memory cannot be shared between the ranks' processes; the updated "
                               "weights are exchanged by NCCL broadcasts")
                self.exchange = "nccl"

    def _alloc_global_results(self, n: int) -> None:
        """One float64 buffer of per-block results indexed by global block: sums [n, NSUMS],
        flags and the 4 status words [n + 4], statistics [n, NSTATS] (integers and fp32 values are
        exact in fp64, and each block's entries are nonzero on its owner only, so a sum over the
        group gathers them)."""
        a = n * _lib.NSUMS
        b = a + n + 4
        self.g_state = torch.zeros(b + n * _lib.NSTATS, dtype=torch.float64, device=self.device)
        self.g_sums = self.g_state[:a].view(n, _lib.NSUMS)
        self.g_flags = self.g_state[a:b]
        self.g_stats = self.g_state[b:].view(n, _lib.NSTATS)
        self.g_bytes = 8 * self.g_state.numel()

    # ------------------------------------------------------------------ exchange hooks
    def _after_chunk(self, ch, stream) -> None:
        if self._peer is not None:
            ready = torch.cuda.Event()
            ready.record(stream)
            self._peer.push(ch.blocks, ready)

    def _after_class(self, class_key) -> None:
        """The blocks of `class_key` are final on their owners (their GEMMs are queued)."""
        if self.world <= 1 or self.exchange != "nccl":
            return
        if os.environ.get("MUZO_COLLECTIVES", "end") == "class":
            self._handles.append(self._broadcast(self._class_blocks([class_key])))
        else:
            self._pending.append(class_key)

    def _class_blocks(self, class_keys) -> list:
        return [b for ck in class_keys for b in self.blocks if (b.rows, b.cols, self._code(b)) == ck]

    def _broadcast(self, blocks):
        """Broadcast `blocks` from their owners in one NCCL group (async)."""
        manager = getattr(dist, "_coalescing_manager", None)
        if dist.get_backend(self.group) == "nccl" and manager is not None:
            with manager(group=self.group, device=self.device, async_ops=True) as cm:
                for b in blocks:
                    dist.broadcast(b.tensor, src=self._global_ranks[self.owner[b.index]], group=self.group)
            return cm
        return [dist.broadcast(b.tensor, src=self._global_ranks[self.owner[b.index]], group=self.group,
                               async_op=True) for b in blocks]

    @staticmethod
    def _code(b) -> int:
        return _lib.dtype_code(b.dtype)

    def _finish_collectives(self) -> None:
        """Scatter this rank's per-block results into the global buffers, sum them over the group
        (after every push of this rank: in the peer exchange this all-reduce is the barrier that
        tells each rank its replica is complete), and make the compute stream wait for it."""
        if self.exchange == "nccl":
            pending, self._pending = self._pending, []
            if pending:
                self._handles.append(self._broadcast(self._class_blocks(pending)))
        compute = torch.cuda.current_stream(self.device) if self.device.type == "cuda" else None
        if compute is not None:
            self._mark("exchange", True)
        self.scatter_owned_results()
        if compute is not None:
            self.comm_stream.wait_stream(compute)
            if self._peer is not None:
                self._peer.join(self.comm_stream)
            with torch.cuda.stream(self.comm_stream):
                self.reduce_results()
            compute.wait_stream(self.comm_stream)
            self._mark("exchange", False)
        else:
            self.reduce_results()
        handles, self._handles = self._handles, []
        for h in handles:
            for w in (h if isinstance(h, list) else [h]):
                w.wait()

    def scatter_owned_results(self) -> None:
        n_owned = self.n_slots
        n = len(self.blocks)
        self.g_state.zero_()
        if n_owned:
            sums = self.state[:self.sums_bytes].view(torch.float64).view(-1, _lib.NSUMS)[:n_owned]
            flags = self.state[self.flags_off:self.flags_off + 4 * (max(n_owned, 1) + 4)].view(torch.int32)
            stats = self.state[self.stats_off:self.state_bytes].view(torch.float32).view(-1, _lib.NSTATS)[:n_owned]
            self.g_sums.index_copy_(0, self.owned_global, sums)
            self.g_flags[:n].index_copy_(0, self.owned_global, flags[:n_owned].to(torch.float64))
            self.g_stats.index_copy_(0, self.owned_global, stats.to(torch.float64))
            self.g_flags[n:n + 4].copy_(flags[n_owned:n_owned + 4].to(torch.float64))

    def reduce_results(self) -> None:
        """Sum the global per-block buffer over the group (one all-reduce)."""
        if self.world > 1:
            dist.all_reduce(self.g_state, group=self.group)

    def _read_results(self, lr32: float) -> dict[int, dict[str, float]]:
        host = self.g_state.cpu().numpy()
        n = len(self.blocks)
        a, b = n * _lib.NSUMS, n * _lib.NSUMS + n + 4
        sums = host[:a].reshape(n, _lib.NSUMS)
        flags = host[a:b].astype(np.int64)
        stats = host[b:].astype(np.float32).reshape(n, _lib.NSTATS)
        return self._stats_from(sums, flags[:n], stats, int(flags[n]), [(b, b.index) for b in self.blocks], lr32)

    def gather_stats(self, per_block: dict[int, dict]) -> dict[int, dict]:
        """The per-block statistics of every block (already combined over the group by the step)."""
        return per_block

    def close(self) -> None:
        if self._peer is not None:
            self._peer.close()
            self._peer = None
