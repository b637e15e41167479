"""Sharded step over the ranks of a torch.distributed process group (one process per GPU).

Every rank keeps a full replica of the selected weights. Perturbation needs no communication:
the noise of a block is a pure function of (seed, name, shape, block index), so all ranks
perturb their replicas identically. The step is partitioned: blocks are assigned to ranks by
Newton-Schulz FLOPs (LPT greedy, identical on every rank); each rank rebuilds, orthogonalises
and applies only its blocks, and once its last GEMM is queued the owners broadcast the updated
blocks with NCCL, all in one group, on NCCL's stream; the compute stream waits for them before
the next use of the weights. Per-block statistics are combined with one small all-reduce.
"""

from __future__ import annotations

import os

import numpy as np
import torch
import torch.distributed as dist

from ._engine import StepEngine


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

    def _after_class(self, class_key) -> None:
        """The blocks of `class_key` are final on their owners (their GEMMs are queued)."""
        if self.world <= 1:
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
        from . import _lib

        return _lib.dtype_code(b.dtype)

    def _finish_collectives(self) -> None:
        """Issue what is still pending and make the current stream wait for every transfer."""
        pending, self._pending = self._pending, []
        if pending:
            self._handles.append(self._broadcast(self._class_blocks(pending)))
        handles, self._handles = self._handles, []
        for h in handles:
            for w in (h if isinstance(h, list) else [h]):
                w.wait()

    def gather_stats(self, per_block: dict[int, dict]) -> dict[int, dict]:
        """Combine the owners' per-block statistics on every rank (sum all-reduce)."""
        n = len(self.blocks)
        host = np.zeros((n, 3), dtype=np.float64)
        for i, st in per_block.items():
            host[i] = (st["update_rms"], st["ratio"], 1.0)
        t = torch.from_numpy(host).to(self.device)
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        host = t.cpu().tolist()
        return {i: {"update_rms": row[0], "ratio": row[1]} for i, row in enumerate(host) if row[2] > 0}
