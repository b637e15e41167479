"""The timeout path of the Newton-Schulz GEMMs, made to run on purpose without faulting anything.

Every wait inside the tcgen05 kernels is bounded. A stall request in status word 3 makes one
role — 1 the TMA producer, 2 the MMA issuer, 3 the epilogue — wait, before its first step, on a
barrier that nothing arrives at; that bounded wait expires and the launch ends through the
timeout path: the status word holds the role's code, the CTAs drain their own copies and MMAs and
free their tensor memory, and the tile scheduler's words are rewound. The next launch on the same
status buffer (status and request cleared) must then run normally and compute the right result.
Through the optimizer the same expiry surfaces as a MuzoError from step(), and the following step
runs normally. Reference recovery paths this mirrors: muzo_clip/muzo_optimizer.py:213-215
(exceptions inside a projection are re-raised after the restore) and newton_schulz.py:63-65.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["wide", "pair", "single"])
def gemm_kernel(request, monkeypatch):
    """The 512 x 768 output runs on the wide pair kernel (256 x 512 tiles, its second tile column
    half empty), on the 256 x 256 pair kernel with MUZO_GEMM_WIDE=0, on one SM with
    MUZO_GEMM_PAIR=0."""
    monkeypatch.setenv("MUZO_GEMM_PAIR", "0" if request.param == "single" else "1")
    monkeypatch.setenv("MUZO_GEMM_WIDE", "1" if request.param == "wide" else "0")
    return request.param


def _update_gemm(L, device, status, sums=None, scales=None, flags=None):
    """X' = a X + B X on a batch of two 512 x 768 matrices (update epilogue); returns (out, ref)."""
    g = torch.Generator(device="cpu").manual_seed(5)
    m, n, batch = 512, 768, 2
    Bm = (torch.randn((batch, m, m), generator=g) * 0.05).to(torch.bfloat16).to(device)
    X = (torch.randn((batch, m, n), generator=g) * 0.05).to(torch.bfloat16).to(device)
    D = torch.zeros_like(X)
    a = np.float32(3.4445)
    L.check(L.lib.muzo_ns_gemm(Bm.data_ptr(), m, m * m, 0, X.data_ptr(), n, m * n, 1, D.data_ptr(), n, m * n,
                               X.data_ptr(), L.EPI_UPDATE, float(a), 0.0, m, n, m, batch, 0,
                               sums, scales, flags, status.data_ptr(), L.stream_ptr(device)), "gemm")
    acc = torch.matmul(Bm.float(), X.float())
    ref = ((float(a) * X.float()).to(torch.bfloat16).float() + acc.to(torch.bfloat16).float()).to(torch.bfloat16)
    return D, ref


@pytest.mark.parametrize("role", [1, 2, 3])
def test_gemm_wait_expiry_reports_drains_and_recovers(device, gemm_kernel, role):
    from muzo_clip_b200 import _lib as L

    status = torch.zeros(4, dtype=torch.int32, device=device)
    status[3] = role
    _update_gemm(L, device, status)
    torch.cuda.synchronize()
    st = status.tolist()
    assert st[0] == role, st          # the stalled role's wait expired first and recorded its code
    assert st[1] == 0 and st[2] == 0, st   # the tile scheduler's words are rewound
    # the context is usable and the next launch on the same buffer is normal
    status.zero_()
    sums = torch.zeros((2, L.NSUMS), dtype=torch.float64, device=device)
    scales = torch.tensor([0.5, 2.0], dtype=torch.float32, device=device)
    flags = torch.zeros(2, dtype=torch.int32, device=device)
    D, ref = _update_gemm(L, device, status, sums.data_ptr(), scales.data_ptr(), flags.data_ptr())
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0, 0, 0]
    err = (D.float() - ref.float()).abs()
    assert float((err > 2.0 ** -7 * ref.float().abs() * 4 + 1e-3).float().mean()) == 0.0
    # the fused sum of squares of the stored result, per matrix
    want = [(D[j].double() * float(scales[j])).square().sum().item() for j in range(2)]
    np.testing.assert_allclose(sums[:, L.SUM_U2].cpu().numpy(), want, rtol=1e-6)
    assert flags.tolist() == [0, 0]


def test_step_raises_on_expired_wait_and_next_step_runs(device):
    """The optimizer surfaces the expired wait as a MuzoError once the step's statistics are
    read; the next step (request cleared) runs through the same engine and buffers."""
    import random

    from muzo_clip_b200 import MuZOClipOptimizer, _lib
    from muzo_clip_b200.muzo_optimizer import HistoryItem

    model = torch.nn.Module()
    model.q_proj = torch.nn.Linear(512, 256, bias=False).to(device)
    opt = MuZOClipOptimizer(model, lr=1e-3, ns_steps=1, min_history=1, seed=3)
    rng = random.Random(2)
    for _ in range(3):
        opt.history.append(HistoryItem(rng.randrange(0, 2**63 - 1), rng.uniform(-3, 3), 0.0, 0.0, 0.0))
    eng = opt._engine_for_step()
    eng.gemm_stall_request = 2
    opt._has_pending_update = True
    with pytest.raises(_lib.MuzoError, match="status 2"):
        opt.step()
    eng.gemm_stall_request = 0
    before = model.q_proj.weight.detach().clone()
    opt._has_pending_update = True
    stats = opt.step()
    assert not stats["skipped"] and stats["updated_param_count"] == 1
    assert bool(torch.isfinite(model.q_proj.weight).all())
    assert not torch.equal(model.q_proj.weight, before)
