"""The exact-accumulation update of a parameter block, and a capture of this build's Newton-Schulz
result — TEST INFRASTRUCTURE.

``exact_block_update`` follows one block through the reference's step (muzo_clip/
muzo_optimizer.py:315-357): the momentum from the reference's own noise path
(``torch_reference.rebuild``), the exact-accumulation Newton-Schulz iteration
(``exact_ns.ns5_exact``) and the oracle's scale / ratio clip / apply / decay arithmetic
(``muzo_oracle.apply_update``). ``capture_ns_outputs`` records the bf16 Newton-Schulz result of
every block as the step engine produces it, just before the update is applied, so a test can
compare the applied update dtype(U) itself rather than the weights it lands on.
"""

from __future__ import annotations

import torch

import muzo_oracle as orc
import torch_reference as tr
from exact_ns import ns5_exact

_DT = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}


def exact_block_update(w0: torch.Tensor, name: str, block_index: int, history, opt, lr: float,
                       distribution: str) -> orc.ApplyResult:
    """ApplyResult (new weights, the applied update .u, ratio, clip) of one block whose weights
    before the step are w0."""
    M = tr.rebuild(w0, name, block_index, history, opt.beta_momentum, distribution, opt.normalize_momentum)
    X = ns5_exact(M, opt.ns_steps)
    return orc.apply_update(w0.float().cpu().numpy(), X.cpu().numpy(), lr, opt.muon_scale, opt.update_ratio_clip,
                            opt.weight_decay, _DT[w0.dtype])


def block_update_from_ns(w0: torch.Tensor, x: torch.Tensor, opt, lr: float) -> orc.ApplyResult:
    """The oracle's apply of a given Newton-Schulz result x to weights w0."""
    return orc.apply_update(w0.float().cpu().numpy(), x.float().cpu().numpy(), lr, opt.muon_scale,
                            opt.update_ratio_clip, opt.weight_decay, _DT[w0.dtype])


def capture_ns_outputs(opt) -> dict:
    """Install a hook on the optimizer's step engine; returns the dict that fills with
    {(name, block_index): bf16 Newton-Schulz result} during the next step()."""
    captured: dict = {}

    def hook(blocks, x, stream):
        with torch.cuda.stream(stream):
            for j, b in enumerate(blocks):
                captured[(b.name, b.block_index)] = x[j].clone()

    opt._engine_for_step().ns_output_hook = hook
    return captured


def rel(a, b) -> float:
    import numpy as np

    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
