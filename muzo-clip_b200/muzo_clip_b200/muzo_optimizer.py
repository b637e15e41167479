"""MuZO-Clip optimizer with the B200 kernel path (mirror of muzo_clip/muzo_optimizer.py).

Same constructor, methods, validation errors, skip logic and returned dicts as the reference
(muzo_optimizer.py:77-504). The host keeps the scalar state (history deque, EMAs, seeds); the
model-sized work — perturbation, momentum rebuild, Newton-Schulz and the update — runs in the
native library through ``_engine.StepEngine``.

Three keyword arguments are additions: ``process_group`` shards the step over the ranks of a
torch.distributed group (each rank rebuilds, orthogonalises and applies the blocks it owns, and
NCCL broadcasts the updated weights; SPSA losses are averaged over the group and QK-Clip maxima
max-reduced, so ranks may feed different batches),
``workspace_bytes`` bounds the Newton-Schulz workspace, and ``noise_cache=True`` keeps the
rounded normal noise of the current projection on the device (one buffer the size of the
selected weights, left out when it would take more than half of the free memory) so that its
-2eps and +eps passes read it back instead of regenerating it; results are bit-identical.
"""

from __future__ import annotations

import logging
import math
import random
from collections import deque
from dataclasses import dataclass
from typing import Callable, Iterable

import torch

from ._engine import StepEngine
from .parameter_filter import (
    DEFAULT_FROZEN_SUBSTRINGS,
    DEFAULT_TRAINABLE_SUBSTRINGS,
    SelectedParameter,
    select_muzo_parameters,
)
from .prng import NoiseDistribution
from .qk_clip import QKClipApplyStats, QKClipController

logger = logging.getLogger(__name__)


@dataclass(frozen=True)
class HistoryItem:
    seed: int
    p: float
    p_raw: float
    loss_plus: float
    loss_minus: float


@dataclass
class ProjectionStats:
    seed: int | None
    loss_plus: float | None
    loss_minus: float | None
    p_raw: float | None
    p_used: float | None
    skipped: bool
    skip_reason: str | None


@dataclass
class StepStats:
    lr: float
    update_rms_mean: float
    update_ratio_max: float
    updated_param_count: int
    skipped: bool
    skip_reason: str | None


def _as_float(value) -> float:
    """Scalar loss of a closure result: ``.loss`` if present, tensor mean, else float()."""
    if hasattr(value, "loss"):
        value = getattr(value, "loss")
    if isinstance(value, torch.Tensor):
        t = value.detach()
        if t.numel() != 1:
            t = t.mean()
        return float(t.float().cpu().item())
    return float(value)


class MuZOClipOptimizer:
    """Muon-style zeroth-order optimizer with seed-replayed momentum, on sm_100a kernels."""

    def __init__(
        self,
        model: torch.nn.Module,
        *,
        lr: float = 1e-5,
        zo_eps: float = 1e-3,
        horizon: int = 8,
        beta_momentum: float = 0.9,
        ns_steps: int = 5,
        weight_decay: float = 0.01,
        p_clip_value: float = 3.0,
        p_ema_beta: float = 0.95,
        update_ratio_clip: float = 0.01,
        distribution: NoiseDistribution = "normal",
        block_rows: int | None = None,
        seed: int = 1,
        rollback: bool = False,
        restore_exact: bool = False,
        min_history: int = 4,
        loss_spike_ratio: float = 2.0,
        trainable_substrings: Iterable[str] = DEFAULT_TRAINABLE_SUBSTRINGS,
        frozen_substrings: Iterable[str] = DEFAULT_FROZEN_SUBSTRINGS,
        normalize_momentum: bool = True,
        muon_scale: float = 0.2,
        enable_qk_clip: bool = False,
        qk_capture_clean_forward: bool = False,
        qk_clip_tau: float = 100.0,
        qk_clip_alpha: float = 0.5,
        process_group=None,
        workspace_bytes: int | None = None,
        noise_cache: bool = False,
    ):
        # argument validation of muzo_optimizer.py:109-122, same messages
        checks = (
            (horizon <= 0, "horizon must be positive"),
            (min_history <= 0, "min_history must be positive"),
            (min_history > horizon, "min_history must be less than or equal to horizon"),
            (zo_eps <= 0, "zo_eps must be positive"),
            (update_ratio_clip <= 0, "update_ratio_clip must be positive"),
            (muon_scale <= 0, "muon_scale must be positive"),
        )
        for failed, message in checks:
            if failed:
                raise ValueError(message)
        if distribution not in ("normal", "rademacher"):
            raise ValueError(f"Unsupported distribution: {distribution}")

        self.model = model
        self.lr = float(lr)
        self.zo_eps = float(zo_eps)
        self.horizon = int(horizon)
        self.beta_momentum = float(beta_momentum)
        self.ns_steps = int(ns_steps)
        self.weight_decay = float(weight_decay)
        self.p_clip_value = float(p_clip_value)
        self.p_ema_beta = float(p_ema_beta)
        self.update_ratio_clip = float(update_ratio_clip)
        self.distribution = distribution
        self.block_rows = block_rows
        self.rollback = bool(rollback)
        self.restore_exact = bool(restore_exact)
        self.min_history = int(min_history)
        self.loss_spike_ratio = float(loss_spike_ratio)
        self.normalize_momentum = bool(normalize_momentum)
        self.muon_scale = float(muon_scale)
        self.qk_capture_clean_forward = bool(qk_capture_clean_forward)
        self.workspace_bytes = workspace_bytes
        self.process_group = process_group
        self.noise_cache = bool(noise_cache)

        self.selected_params: list[SelectedParameter] = select_muzo_parameters(
            model, trainable_substrings=trainable_substrings, frozen_substrings=frozen_substrings
        )
        if not self.selected_params:
            logger.warning("MuZO-Clip selected no parameters with the current filter")
        elif not self.restore_exact and self._has_low_precision_selected_params():
            logger.warning(
                "MuZO-Clip selected fp16/bf16 parameters while restore_exact=False; "
                "+eps/-2eps/+eps perturb restore is not numerically exact in low precision. "
                "This avoids CPU snapshots and is the intended LLM default."
            )
        if self.rollback:
            logger.warning("rollback=True snapshots selected params to CPU; avoid this for LLM-scale runs.")
        if self.restore_exact:
            logger.warning("restore_exact=True snapshots selected params to CPU; avoid this for LLM-scale runs.")

        self.history: deque[HistoryItem] = deque(maxlen=self.horizon)
        self.p_abs_ema: float = 0.0
        self.loss_ema: float | None = None
        self.bad_step_count: int = 0
        self.lr_scale: float = 1.0
        self._rng = random.Random(int(seed))
        self._has_pending_update = False
        self._last_step_updated = False
        self._engine: StepEngine | None = None
        self._snapshot_bufs: list[torch.Tensor] | None = None

        self.qk_clip: QKClipController | None = None
        if enable_qk_clip:
            self.qk_clip = QKClipController(model, tau=qk_clip_tau, alpha=qk_clip_alpha,
                                            process_group=process_group)

    # ------------------------------------------------------------------ public API
    @property
    def current_lr(self) -> float:
        return self.lr * self.lr_scale

    def selected_parameter_names(self) -> list[str]:
        return [item.name for item in self.selected_params]

    def persistent_tensor_state(self) -> list[torch.Tensor]:
        """Persistent non-parameter tensors owned by the optimizer (the QK-Clip maxima)."""
        if self.qk_clip is None:
            return []
        return list(self.qk_clip.persistent_tensors())

    @torch.no_grad()
    def estimate_projection(self, loss_closure: Callable[[], object]) -> dict[str, object]:
        """SPSA +eps / -eps projection; appends the scalar to the history (muzo_optimizer.py:190-268)."""

        seed = self._sample_seed()
        self._clear_qk_clip_capture()
        snapshot = self._snapshot_selected_params() if (self.rollback or self.restore_exact) else None
        displacement = 0
        try:
            self._perturb_selected(seed, scaling_factor=1.0)
            displacement = 1
            loss_plus = self._call_loss(loss_closure)
            self._perturb_selected(seed, scaling_factor=-2.0)
            displacement = -1
            loss_minus = self._call_loss(loss_closure)
            if self.restore_exact and snapshot is not None:
                self._restore_snapshot(snapshot)
            else:
                self._perturb_selected(seed, scaling_factor=1.0)
            displacement = 0
        except Exception:
            self._restore_after_failed_projection(seed, displacement, snapshot)
            raise

        loss_plus, loss_minus = self._reduce_losses(loss_plus, loss_minus)
        p_raw = (loss_plus - loss_minus) / (2.0 * self.zo_eps)
        skip_reason = self._projection_skip_reason(loss_plus, loss_minus, p_raw)
        if skip_reason is not None:
            if snapshot is not None:
                self._restore_snapshot(snapshot)
            if self.qk_clip is not None:
                self.qk_clip.clear()
            self.bad_step_count += 1
            self.lr_scale = max(self.lr_scale * 0.5, 1e-4)
            self._has_pending_update = False
            return ProjectionStats(seed, loss_plus, loss_minus, p_raw, None, True, skip_reason).__dict__

        abs_p = abs(float(p_raw))
        if self.p_abs_ema == 0.0:
            self.p_abs_ema = abs_p
        else:
            self.p_abs_ema = self.p_ema_beta * self.p_abs_ema + (1.0 - self.p_ema_beta) * abs_p
        p_norm = float(p_raw) / (self.p_abs_ema + 1e-12)
        p_used = max(-self.p_clip_value, min(self.p_clip_value, p_norm))

        self.history.append(HistoryItem(int(seed), float(p_used), float(p_raw), float(loss_plus), float(loss_minus)))
        self._has_pending_update = True
        self._update_loss_ema(0.5 * (float(loss_plus) + float(loss_minus)))
        if self.qk_clip is not None and self.qk_capture_clean_forward:
            with self.qk_clip.capture():
                self._call_loss(loss_closure)
        return ProjectionStats(seed, loss_plus, loss_minus, p_raw, p_used, False, None).__dict__

    @torch.no_grad()
    def step(self) -> dict[str, object]:
        """Rebuild the momentum from the seed history and apply the Muon-style update
        (muzo_optimizer.py:270-371)."""

        skip = None
        if not self._has_pending_update:
            skip = "no successful pending projection"
        elif not self.history:
            skip = "empty projection history"
        elif len(self.history) < self.min_history:
            skip = f"waiting for min_history={self.min_history}"
        if skip is not None:
            self._has_pending_update = False
            self._last_step_updated = False
            self._clear_qk_clip_capture()
            return StepStats(self.current_lr, 0.0, 0.0, 0, True, skip).__dict__

        lr = self.current_lr
        per_block = self._engine_for_step().run_step(self.history, lr) if self.selected_params else {}
        per_block = self._gather_block_stats(per_block)
        update_rms_values = [per_block[i]["update_rms"] for i in sorted(per_block)]
        update_ratio_max = 0.0
        for i in sorted(per_block):
            update_ratio_max = max(update_ratio_max, per_block[i]["ratio"])
        updated_param_count = len(per_block)

        self._has_pending_update = False
        self._last_step_updated = updated_param_count > 0
        mean_update_rms = sum(update_rms_values) / len(update_rms_values) if update_rms_values else 0.0
        return StepStats(lr, mean_update_rms, update_ratio_max, updated_param_count, False, None).__dict__

    @torch.no_grad()
    def apply_qk_clip_if_available(self) -> dict[str, object]:
        if self.qk_clip is None:
            return QKClipApplyStats(False, False, False, "QK-Clip controller is not enabled", 0.0, 0).__dict__
        if not self._last_step_updated:
            self.qk_clip.clear()
            return QKClipApplyStats(
                False, False, False, "QK-Clip skipped because the last MuZO step did not update weights", 0.0, 0
            ).__dict__
        self._last_step_updated = False
        return self.qk_clip.apply().__dict__

    @torch.no_grad()
    def probe_and_apply_qk_clip(self, clean_forward_closure: Callable[[], object], *,
                                force_eager: bool = True) -> dict[str, object]:
        """One clean forward that records the per-head max pre-softmax logit, then QK-Clip
        (muzo_optimizer.py:397-426)."""
        if self.qk_clip is None:
            return QKClipApplyStats(False, False, False, "QK-Clip controller is not enabled", 0.0, 0).__dict__

        def wrapped_forward() -> float:
            return self._call_loss(clean_forward_closure)

        return self.qk_clip.probe(wrapped_forward, force_eager=force_eager).__dict__

    # ------------------------------------------------------------------ resume
    def state_dict(self) -> dict[str, object]:
        """Everything needed to resume the optimizer exactly: the seed history that defines the
        momentum, the scalar EMAs and back-off, the seed generator's state and the pending flags.
        No model-sized tensor is stored (the momentum is rebuilt from the history)."""
        return {
            "format": "muzo_clip_b200.state.v1",
            "history": [dict(h.__dict__) for h in self.history],
            "horizon": self.horizon,
            "p_abs_ema": self.p_abs_ema,
            "loss_ema": self.loss_ema,
            "bad_step_count": self.bad_step_count,
            "lr_scale": self.lr_scale,
            "rng_state": self._rng.getstate(),
            "has_pending_update": self._has_pending_update,
            "last_step_updated": self._last_step_updated,
            "selected_parameter_names": self.selected_parameter_names(),
        }

    def load_state_dict(self, state: dict[str, object]) -> None:
        """Restore a state_dict() of an optimizer over the same selected parameters."""
        if state.get("format") != "muzo_clip_b200.state.v1":
            raise ValueError("not a muzo_clip_b200 optimizer state")
        if list(state["selected_parameter_names"]) != self.selected_parameter_names():
            raise ValueError("the state was saved for a different set of selected parameters")
        self.history = deque((HistoryItem(**h) for h in state["history"]), maxlen=self.horizon)
        self.p_abs_ema = float(state["p_abs_ema"])
        self.loss_ema = None if state["loss_ema"] is None else float(state["loss_ema"])
        self.bad_step_count = int(state["bad_step_count"])
        self.lr_scale = float(state["lr_scale"])
        rng_state = state["rng_state"]
        if isinstance(rng_state, list):  # after a JSON round trip
            rng_state = (rng_state[0], tuple(rng_state[1]), rng_state[2])
        self._rng.setstate(rng_state)
        self._has_pending_update = bool(state["has_pending_update"])
        self._last_step_updated = bool(state["last_step_updated"])

    # ------------------------------------------------------------------ internals
    def _engine_for_step(self) -> StepEngine:
        if self._engine is None or not self._engine.matches(self):
            if self.process_group is not None:
                from .distributed import ShardedStepEngine

                self._engine = ShardedStepEngine(self, self.process_group)
            else:
                self._engine = StepEngine(self)
        return self._engine

    def _sample_seed(self) -> int:
        return self._rng.randrange(0, (1 << 63) - 1)

    def _has_low_precision_selected_params(self) -> bool:
        return any(s.param.dtype in (torch.float16, torch.bfloat16) for s in self.selected_params)

    @torch.no_grad()
    def _perturb_selected(self, seed: int, scaling_factor: float) -> None:
        if not self.selected_params:
            return
        self._engine_for_step().perturb(seed, float(scaling_factor) * self.zo_eps)

    def _call_loss(self, loss_closure: Callable[[], object]) -> float:
        self.model.eval()
        with torch.no_grad():
            return _as_float(loss_closure())

    def _reduce_losses(self, loss_plus: float, loss_minus: float) -> tuple[float, float]:
        """Average the two SPSA losses over the process group so every rank derives the same p."""
        if self.process_group is None:
            return loss_plus, loss_minus
        import torch.distributed as dist

        world = dist.get_world_size(self.process_group)
        if world <= 1:
            return loss_plus, loss_minus
        device = self._engine_for_step().device
        t = torch.tensor([loss_plus, loss_minus], dtype=torch.float64, device=device)
        dist.all_reduce(t, group=self.process_group)
        t /= world
        lp, lm = t.tolist()
        return float(lp), float(lm)

    def _gather_block_stats(self, per_block: dict[int, dict]) -> dict[int, dict]:
        if self.process_group is None:
            return per_block
        return self._engine_for_step().gather_stats(per_block)

    def _projection_skip_reason(self, loss_plus: float, loss_minus: float, p_raw: float) -> str | None:
        for name, value in (("loss_plus", loss_plus), ("loss_minus", loss_minus), ("p_raw", p_raw)):
            if not math.isfinite(float(value)):
                return f"{name} is non-finite"
        if self.loss_ema is not None:
            threshold = self.loss_spike_ratio * max(abs(self.loss_ema), 1e-12)
            if float(loss_plus) > threshold:
                return "loss_plus exceeded loss spike threshold"
            if float(loss_minus) > threshold:
                return "loss_minus exceeded loss spike threshold"
        return None

    def _update_loss_ema(self, loss: float) -> None:
        self.loss_ema = float(loss) if self.loss_ema is None else 0.95 * self.loss_ema + 0.05 * float(loss)

    def _clear_qk_clip_capture(self) -> None:
        if self.qk_clip is not None:
            self.qk_clip.clear()

    @torch.no_grad()
    def _snapshot_selected_params(self):
        """Host copy of every selected parameter for `rollback` / `restore_exact`
        (muzo_optimizer.py:482-483). The copies land in page-locked buffers allocated on first use
        and reused afterwards, as asynchronous device-to-host copies on the current stream: the
        perturbation kernels launched next on that stream start after the copies have read the
        weights, so the host never waits. Without page-locked memory the buffers are pageable and
        the copies synchronous."""
        if self._snapshot_bufs is None:
            bufs = []
            for s in self.selected_params:
                try:
                    bufs.append(torch.empty(s.param.shape, dtype=s.param.dtype, pin_memory=True))
                except RuntimeError:
                    bufs.append(torch.empty(s.param.shape, dtype=s.param.dtype))
            self._snapshot_bufs = bufs
        snapshot = []
        for s, buf in zip(self.selected_params, self._snapshot_bufs):
            buf.copy_(s.param.detach(), non_blocking=True)
            snapshot.append((s.param, buf))
        return snapshot

    @torch.no_grad()
    def _restore_snapshot(self, snapshot) -> None:
        """Copy the snapshot back (muzo_optimizer.py:486-488), host-to-device on the current stream."""
        for param, saved in snapshot:
            param.data.copy_(saved, non_blocking=True)

    @torch.no_grad()
    def _restore_after_failed_projection(self, seed: int, displacement: int, snapshot) -> None:
        if snapshot is not None:
            self._restore_snapshot(snapshot)
        elif displacement == 1:
            self._perturb_selected(seed, scaling_factor=-1.0)
        elif displacement == -1:
            self._perturb_selected(seed, scaling_factor=1.0)
        if self.qk_clip is not None:
            self.qk_clip.clear()
