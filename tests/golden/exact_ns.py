"""Exact-accumulation Newton-Schulz in torch float64 — TEST INFRASTRUCTURE.

The same iteration as ``muzo_oracle.ns5_bf16(exact=True)``: the reference's bf16 op sequence
(muzo_clip/newton_schulz.py:44-58) with every GEMM accumulated in float64 and every GEMM and
element-wise result rounded to fp32 and then to bf16. It is the accumulation-order-free result
that every bf16 implementation approximates (cuBLAS's and the tcgen05 kernels' alike), written
with torch so that it runs on the GPU at the full Llama-3-8B and 8192 x 28672 shapes, where the
numpy oracle would take minutes. ``tests/test_oracle_cpu.py`` checks it against the numpy oracle
on CPU tensors.
"""

from __future__ import annotations

import torch

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def _bf(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def _f32(v: float) -> float:
    return float(torch.tensor(v, dtype=torch.float32))


@torch.no_grad()
def ns5_exact(G: torch.Tensor, steps: int = 5) -> torch.Tensor:
    """fp32 result of the exact-accumulation bf16 iteration on a 2-D tensor, in G's layout;
    zeros for a zero or non-finite input or a non-finite result (newton_schulz.py:35-43, 63-65)."""
    g = G.to(torch.float32)
    zeros = torch.zeros_like(g)
    if not bool(torch.isfinite(g).all()):
        return zeros
    if not float(g.double().square().sum()) > 0.0:
        return zeros
    a, b, c = (_f32(v) for v in NS_COEFFS)
    x = _bf(g)
    transposed = g.shape[0] > g.shape[1]
    if transposed:
        x = x.T.contiguous()
    nrm = x.double().square().sum().sqrt().to(torch.float32)
    x = _bf(x / (nrm + torch.tensor(1e-7, dtype=torch.float32, device=x.device)))

    def mm(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
        return (p.double() @ q.double()).to(torch.float32)

    for _ in range(int(steps)):
        A = _bf(mm(x, x.T))
        AA = _bf(mm(A, A))
        B = _bf(_bf(b * A) + _bf(c * AA))
        del AA
        BX = _bf(mm(B, x))
        x = _bf(_bf(a * x) + BX)
        del A, B, BX
    if transposed:
        x = x.T.contiguous()
    if not bool(torch.isfinite(x).all()):
        return zeros
    return x
