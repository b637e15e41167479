"""Resume through the real kernels: an optimizer rebuilt from a JSON round trip of state_dict()
continues bit-identically to the run that was never interrupted.

The reference keeps its optimizer state in memory only (muzo_clip/muzo_optimizer.py:162-169,
182-188); state_dict() / load_state_dict() carry the seed history that defines the momentum, the
EMAs, the learning-rate back-off, the seed generator and the pending flags.
"""

from __future__ import annotations

import copy
import json

import pytest
import torch

pytestmark = pytest.mark.gpu


class _Mats(torch.nn.Module):
    def __init__(self, device, dtype):
        super().__init__()
        g = torch.Generator(device="cpu").manual_seed(21)
        self.layers = torch.nn.ModuleList()
        for r, c in ((256, 512), (688, 256), (64, 128)):
            m = torch.nn.Module()
            m.q_proj = torch.nn.Linear(c, r, bias=False)
            m.q_proj.weight.data = (torch.randn((r, c), generator=g) * 0.02).to(dtype=dtype, device=device)
            self.layers.append(m)


def _loss(model) -> float:
    # deterministic on one device: a function of the weights only
    return float(sum(p.float().square().sum() for p in model.parameters()).item()) * 1e-3 + 1.0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("noise_cache", [False, True])
def test_resume_from_state_dict_is_bit_identical(device, dtype, noise_cache):
    from muzo_clip_b200 import MuZOClipOptimizer

    kw = dict(lr=1e-3, horizon=4, min_history=2, seed=77, noise_cache=noise_cache)
    model = _Mats(device, dtype)
    opt = MuZOClipOptimizer(model, **kw)

    def run(o, m, n):
        out = []
        for _ in range(n):
            out.append(o.estimate_projection(lambda: _loss(m)))
            out.append(o.step())
        return out

    first = run(opt, model, 3)
    state = json.loads(json.dumps(opt.state_dict()))
    resumed_model = copy.deepcopy(model)
    tail = run(opt, model, 3)

    fresh = MuZOClipOptimizer(resumed_model, **kw)
    fresh.load_state_dict(state)
    tail2 = run(fresh, resumed_model, 3)

    assert any(not s.get("skipped", True) for s in first + tail if "updated_param_count" in s)
    assert tail == tail2
    for (n, p), (_, q) in zip(model.named_parameters(), resumed_model.named_parameters()):
        assert torch.equal(p, q), n
    assert json.loads(json.dumps(fresh.state_dict())) == json.loads(json.dumps(opt.state_dict()))
