"""QK-Clip on B200 (mirror of muzo_clip/qk_clip.py).

The reference records the pre-softmax logits of eager attention by patching ``F.softmax`` and
reduces each to a per-head max with a host sync per layer (qk_clip.py:173-196). Here:

* ``probe(force_eager=True)`` on a transformers model switches the attention modules to a probe
  attention function registered with transformers' AttentionInterface. It receives the
  post-RoPE query and key states and computes the per-head maximum of the eager logits
  ``bf16(bf16(q.k) * scaling)`` (causal, GQA) with the library's tcgen05 max-logit kernel — no
  S x S logits are materialised — and returns the attention output of SDPA.
* Other eager attention code is still captured at ``softmax`` (the reference's mechanism); its
  logits are reduced on the GPU by the library's per-head max kernel.
* Maxima stay on the device until ``apply()``, which reads them in one copy and scales the q/k
  projection rows with the library's row-scaling kernel. Statistics and the GQA grouping rules
  follow qk_clip.py:198-322.
* With a ``process_group`` (data-parallel ranks, each capturing on its own batch), ``apply()``
  first takes the per-head maxima's maximum over the group, so every rank clips its replica
  with the same factors and the replicas stay identical.
"""

from __future__ import annotations

import contextlib
import logging
from dataclasses import dataclass
from typing import Any, Callable, Iterator

import numpy as np
import torch
import torch.nn.functional as F

from . import _qk

logger = logging.getLogger(__name__)

PROBE_ATTENTION = "muzo_qk_probe"
CAPTURE_ATTENTION = "muzo_qk_sdpa"


def use_qk_capture_attention(model: torch.nn.Module) -> str:
    """Make ``model`` (a transformers model) train with the QK-capture attention: SDPA for the
    output and gradients, plus the library's max-logit kernel on the same query/key states
    while a QK-Clip capture is active — e.g. the clean forward of
    ``MuZOClipOptimizer(..., enable_qk_clip=True, qk_capture_clean_forward=True)`` — so exact
    per-head maxima are collected without eager attention and without a separate probe. Outside
    a capture the attention is SDPA alone. Returns the implementation name."""
    impl = _qk.ensure_training_registered()
    seen: list[Any] = []
    for module in model.modules():
        config = getattr(module, "config", None)
        if config is None or any(config is c for c in seen):
            continue
        seen.append(config)
        if hasattr(config, "_attn_implementation"):
            config._attn_implementation = impl
    if not seen:
        raise ValueError("use_qk_capture_attention expects a transformers model (no config found)")
    return impl


@dataclass
class QKClipApplyStats:
    enabled: bool
    exact_logits: bool
    fallback_used: bool
    disabled_reason: str | None
    qk_smax_max: float
    qk_clip_count: int


class QKClipController:
    """Capture per-head pre-softmax maxima and apply QK-Clip to q/k projections."""

    def __init__(self, model: torch.nn.Module, tau: float = 100.0, alpha: float = 0.5, process_group=None):
        self.model = model
        self.tau = float(tau)
        self.alpha = float(alpha)
        self.process_group = process_group
        self.modules: dict[str, torch.nn.Module] = {}
        self._names_by_id: dict[int, str] = {}
        self._handles: list[Any] = []
        self._module_stack: list[str] = []
        self._captured_smax: dict[str, torch.Tensor] = {}   # device fp32 [heads]
        self._warned_unavailable = False
        self._installed = False
        self._install_hooks()

    @property
    def installed(self) -> bool:
        return self._installed

    def close(self) -> None:
        for handle in self._handles:
            handle.remove()
        self._handles.clear()
        self._installed = False

    # ------------------------------------------------------------------ hooks
    def _install_hooks(self) -> None:
        """Attention modules are those with 2-D q_proj and k_proj weights (qk_clip.py:57-74)."""
        for name, module in self.model.named_modules():
            q_proj = getattr(module, "q_proj", None)
            k_proj = getattr(module, "k_proj", None)
            ok = (
                q_proj is not None and k_proj is not None
                and hasattr(q_proj, "weight") and hasattr(k_proj, "weight")
                and q_proj.weight.ndim == 2 and k_proj.weight.ndim == 2
            )
            if not ok:
                continue
            self.modules[name] = module
            self._names_by_id[id(module)] = name
            self._handles.append(module.register_forward_pre_hook(self._make_pre_hook(name)))
            self._handles.append(module.register_forward_hook(self._make_post_hook(name)))
        self._installed = bool(self.modules)
        if not self._installed:
            logger.warning("QK-Clip disabled because no q_proj/k_proj attention modules were found")

    def _make_pre_hook(self, name: str):
        def hook(_module, _inputs) -> None:
            self._module_stack.append(name)

        return hook

    def _make_post_hook(self, name: str):
        def hook(_module, _inputs, _outputs) -> None:
            if self._module_stack and self._module_stack[-1] == name:
                self._module_stack.pop()
            elif name in self._module_stack:
                self._module_stack.remove(name)

        return hook

    # ------------------------------------------------------------------ capture
    def _record(self, module_name: str, per_head: torch.Tensor, valid: torch.Tensor | None) -> None:
        """Merge a device per-head max into the running max of ``module_name``; ``valid`` (device
        int32) gates the merge so that a capture with non-finite logits is dropped."""
        prev = self._captured_smax.get(module_name)
        if prev is None:
            prev = torch.full_like(per_head, float("-inf"))
            self._captured_smax[module_name] = prev
        _qk.merge_max(prev, per_head, valid)

    def _maybe_record_softmax_input(self, input_tensor, args, kwargs) -> None:
        """Softmax-input capture of qk_clip.py:173-196, reduced on the GPU."""
        if not self._module_stack:
            return
        if not isinstance(input_tensor, torch.Tensor) or input_tensor.ndim != 4:
            return
        dim = kwargs.get("dim", args[0] if args else None)
        if dim not in (-1, input_tensor.ndim - 1):
            return
        if input_tensor.device.type != "cuda":
            return
        per_head, valid = _qk.logits_head_max(input_tensor.detach())
        self._record(self._module_stack[-1], per_head, valid)

    def record_qk(self, module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor, scaling: float,
                  causal: bool, attention_mask: torch.Tensor | None) -> None:
        """Per-head max logit of an attention call from its query/key states (probe path)."""
        name = self._names_by_id.get(id(module))
        if name is None and self._module_stack:
            name = self._module_stack[-1]
        if name is None:
            return
        per_head, valid = _qk.qk_head_max(query, key, scaling, causal, attention_mask)
        self._record(name, per_head, valid)

    def module_name(self, module: torch.nn.Module) -> str | None:
        """The capture name of an attention module (or of the innermost one being run)."""
        name = self._names_by_id.get(id(module))
        if name is None and self._module_stack:
            name = self._module_stack[-1]
        return name

    def record_max(self, name: str, per_head: torch.Tensor, valid: torch.Tensor) -> None:
        """Per-head maxima an attention kernel computed as a side output (fused capture path)."""
        self._record(name, per_head, valid)

    @contextlib.contextmanager
    def capture(self) -> Iterator[None]:
        """Record pre-softmax maxima during forward calls (softmax capture + probe attention)."""
        if not self._installed:
            yield
            return
        original_f_softmax = F.softmax
        original_torch_softmax = torch.softmax
        controller = self

        def patched_f_softmax(input, *args, **kwargs):
            controller._maybe_record_softmax_input(input, args, kwargs)
            return original_f_softmax(input, *args, **kwargs)

        def patched_torch_softmax(input, *args, **kwargs):
            controller._maybe_record_softmax_input(input, args, kwargs)
            return original_torch_softmax(input, *args, **kwargs)

        F.softmax = patched_f_softmax
        torch.softmax = patched_torch_softmax
        token = _qk.set_active_controller(self)
        try:
            yield
        finally:
            _qk.reset_active_controller(token)
            F.softmax = original_f_softmax
            torch.softmax = original_torch_softmax
            self._module_stack.clear()

    @contextlib.contextmanager
    def force_eager_attention(self, enabled: bool = True) -> Iterator[None]:
        """Route attention through the probe implementation for the duration of the probe.

        transformers models read ``config._attn_implementation`` at every forward; it is set to
        the registered probe attention (eager mask, SDPA output, kernel max). Models that choose
        their attention class at construction ignore it and fall back to softmax capture.
        """
        if not enabled:
            yield
            return
        impl = _qk.ensure_probe_registered()
        configs: list[Any] = []
        for module in [self.model, *self.modules.values()]:
            config = getattr(module, "config", None)
            if config is not None and not any(config is c for c in configs):
                configs.append(config)
        saved: list[tuple[Any, str, Any, bool]] = []
        for config in configs:
            for attr in ("_attn_implementation", "attn_implementation"):
                if hasattr(config, attr):
                    saved.append((config, attr, getattr(config, attr), True))
                    try:
                        setattr(config, attr, impl)
                    except Exception:
                        logger.debug("Could not set %s on %s", attr, type(config).__name__)
                else:
                    saved.append((config, attr, None, False))
        try:
            yield
        finally:
            for config, attr, value, existed in reversed(saved):
                try:
                    if existed:
                        setattr(config, attr, value)
                except Exception:
                    logger.debug("Could not restore %s on %s", attr, type(config).__name__)

    @torch.no_grad()
    def probe(self, forward_closure: Callable[[], Any], *, force_eager: bool = True) -> QKClipApplyStats:
        """One clean forward to collect the maxima, then QK-Clip (qk_clip.py:161-171)."""
        self.clear()
        if not self._installed:
            return self.apply()
        with self.force_eager_attention(force_eager):
            with self.capture():
                forward_closure()
        return self.apply()

    # ------------------------------------------------------------------ apply
    @torch.no_grad()
    def reduce_over_group(self) -> None:
        """Replace the captured maxima by their maximum over the process group (every rank must
        call this together). Ranks may have captured different modules: a module captured on any
        rank is present on all afterwards. Two all-reduces: the head counts per module (their
        maximum and, negated, their minimum over the ranks that captured the module, in one
        tensor), then the packed maxima (-inf where a rank has none). Ranks that disagree on a
        module's head count all raise the same ValueError after the first all-reduce, so no rank
        is left waiting in the second."""
        pg = self.process_group
        if pg is None or not self._installed:
            return
        import torch.distributed as dist

        if dist.get_world_size(pg) <= 1:
            return
        names = list(self.modules)  # named_modules order: identical on identical replicas
        first = next(iter(self.modules.values()))
        device = first.q_proj.weight.device
        big = 1 << 40  # stands for "not captured" in the minimum
        have = [self._captured_smax[n].numel() if n in self._captured_smax else None for n in names]
        counts = torch.tensor([c if c is not None else 0 for c in have] + [-(c if c is not None else big) for c in have],
                              dtype=torch.int64, device=device)
        dist.all_reduce(counts, op=dist.ReduceOp.MAX, group=pg)
        both = [int(c) for c in counts.tolist()]
        sizes, smallest = both[:len(names)], [-c for c in both[len(names):]]
        for name, hi, lo in zip(names, sizes, smallest):
            if lo != big and lo != hi:   # every rank sees the same counts and raises alike
                raise ValueError(f"QK-Clip capture of {name}: {lo} heads on one rank, {hi} on another")
        packed = torch.full((max(sum(sizes), 1),), float("-inf"), dtype=torch.float32, device=device)
        off = 0
        for name, k in zip(names, sizes):
            mine = self._captured_smax.get(name)
            if mine is not None:
                packed[off: off + k].copy_(mine.reshape(-1))
            off += k
        dist.all_reduce(packed, op=dist.ReduceOp.MAX, group=pg)
        self._captured_smax.clear()
        off = 0
        for name, k in zip(names, sizes):
            if k:
                self._captured_smax[name] = packed[off: off + k]
            off += k

    @torch.no_grad()
    def apply(self) -> QKClipApplyStats:
        if not self._installed:
            return QKClipApplyStats(False, False, False, "no q_proj/k_proj attention modules found", 0.0, 0)
        self.reduce_over_group()
        if not self._captured_smax:
            reason = "QK-Clip disabled because pre-softmax logits are unavailable. Use attn_implementation='eager'."
            if not self._warned_unavailable:
                logger.warning(reason)
                self._warned_unavailable = True
            return QKClipApplyStats(False, False, False, reason, 0.0, 0)

        names = list(self._captured_smax)
        _qk.check_attention_status(self._captured_smax[names[0]].device)
        host = _qk.to_host([self._captured_smax[n] for n in names])  # one device-to-host copy
        fallback_used = False
        clip_count = 0
        smax_max = 0.0
        jobs: list = []   # row scalings, launched together (their factors in one upload)
        for name, per_head in zip(names, host):
            module = self.modules.get(name)
            if module is None:
                continue
            smax_max = max(smax_max, float(per_head.max()))
            needs_clip = per_head > np.float32(self.tau)
            if not needs_clip.any():
                continue
            gamma = np.minimum(np.float32(self.tau) / np.maximum(per_head, np.float32(1e-12)),
                               np.float32(1.0)).astype(np.float32)
            clipped, used_fallback = self._scale_qk(module.q_proj.weight, module.k_proj.weight, gamma, needs_clip,
                                                    jobs)
            clip_count += clipped
            fallback_used = fallback_used or used_fallback
        _qk.scale_rows_many(jobs)
        self._captured_smax.clear()
        return QKClipApplyStats(True, True, fallback_used, None, smax_max, clip_count)

    def persistent_tensors(self) -> list[torch.Tensor]:
        return list(self._captured_smax.values())

    def clear(self) -> None:
        self._captured_smax.clear()

    @torch.no_grad()
    def _scale_qk(self, q_weight: torch.Tensor, k_weight: torch.Tensor, gamma: np.ndarray,
                  needs_clip: np.ndarray, jobs: list) -> tuple[int, bool]:
        """Per-head q rows * gamma^alpha, per kv-group k rows * (min gamma)^(1-alpha)
        (qk_clip.py:262-310); whole-matrix fallback when the head layout does not divide. The
        row scalings are appended to ``jobs``."""
        hq = int(gamma.size)
        if hq <= 0 or q_weight.ndim != 2 or k_weight.ndim != 2 or q_weight.shape[0] % hq != 0:
            return self._scale_qk_fallback(q_weight, k_weight, gamma, jobs)
        hd = q_weight.shape[0] // hq
        if hd <= 0 or k_weight.shape[0] % hd != 0:
            return self._scale_qk_fallback(q_weight, k_weight, gamma, jobs)
        hk = k_weight.shape[0] // hd
        if hk <= 0 or hq % hk != 0:
            return self._scale_qk_fallback(q_weight, k_weight, gamma, jobs)
        q_factors = _qk.pow_factors(gamma, self.alpha, q_weight.dtype)
        jobs.append((q_weight, hq, hd, q_factors, needs_clip))
        group = hq // hk
        k_gamma = gamma.reshape(hk, group).min(axis=1)
        k_mask = needs_clip.reshape(hk, group).any(axis=1)
        k_factors = _qk.pow_factors(k_gamma, 1.0 - self.alpha, k_weight.dtype)
        jobs.append((k_weight, hk, hd, k_factors, k_mask))
        return int(needs_clip.sum()) + int(k_mask.sum()), False

    @torch.no_grad()
    def _scale_qk_fallback(self, q_weight: torch.Tensor, k_weight: torch.Tensor,
                           gamma: np.ndarray, jobs: list) -> tuple[int, bool]:
        g = np.minimum(gamma.min(), np.float32(1.0)).astype(np.float32).reshape(1)
        one = np.ones(1, dtype=bool)
        jobs.append((q_weight, 1, q_weight.shape[0], _qk.pow_factors(g, self.alpha, q_weight.dtype), one))
        jobs.append((k_weight, 1, k_weight.shape[0], _qk.pow_factors(g, 1.0 - self.alpha, k_weight.dtype), one))
        return 2, True
