"""Newton-Schulz orthogonalisation on B200 tensor cores (mirror of muzo_clip/newton_schulz.py).

The quintic iteration ``A = X X^T; B = b A + c A A; X = a X + B X`` (newton_schulz.py:55-58) runs
as three batched tcgen05 GEMMs per step with the element-wise terms fused into their epilogues,
in bf16 with fp32 accumulation and the reference's per-op bf16 rounding. Tall matrices are not
transposed in memory: the GEMMs read them through MN-major operand descriptors and write the
result back in the matrix's own layout.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

logger = logging.getLogger(__name__)

# Quintic coefficients (a, b, c) of newton_schulz.py:45 (from KellerJordan/Muon).
NS_COEFFS = (3.4445, -4.7750, 2.0315)


def _round8(v: int) -> int:
    return (v + 7) // 8 * 8


@dataclass
class NSBuffers:
    """Workspace of one batch of same-shape matrices.

    ``x`` holds two ping-pong copies [2, batch, rows, ld] of the iterate in the matrix's own
    layout; ``a`` and ``b`` hold [batch, m, ldm] with m = min(rows, cols).
    """

    rows: int
    cols: int
    batch: int
    ld: int
    ldm: int
    x: torch.Tensor
    a: torch.Tensor
    b: torch.Tensor

    @property
    def m(self) -> int:
        return min(self.rows, self.cols)

    def x_slot(self, parity: int) -> torch.Tensor:
        return self.x[parity]


def _align256(v: int) -> int:
    return (v + 255) // 256 * 256


def ns_workspace_bytes(rows: int, cols: int, batch: int) -> int:
    """Bytes of the workspace of ``batch`` rows x cols matrices (see NSBuffers)."""
    ld, m = _round8(cols), min(rows, cols)
    ldm = _round8(m)
    return _align256(2 * batch * rows * ld * 2) + 2 * _align256(batch * m * ldm * 2)


def ns_buffers_in(raw: torch.Tensor, rows: int, cols: int, batch: int) -> NSBuffers:
    """NSBuffers carved out of a flat uint8 device buffer of at least ns_workspace_bytes."""
    ld, m = _round8(cols), min(rows, cols)
    ldm = _round8(m)
    xb = 2 * batch * rows * ld * 2
    mb = batch * m * ldm * 2
    off_a = _align256(xb)
    off_b = off_a + _align256(mb)
    if raw.numel() < off_b + mb:
        raise ValueError("workspace too small")
    x = raw[:xb].view(torch.bfloat16).view(2, batch, rows, ld)
    a = raw[off_a:off_a + mb].view(torch.bfloat16).view(batch, m, ldm)
    b = raw[off_b:off_b + mb].view(torch.bfloat16).view(batch, m, ldm)
    return NSBuffers(rows, cols, batch, ld, ldm, x, a, b)


def allocate_ns_buffers(rows: int, cols: int, batch: int, device: torch.device) -> NSBuffers:
    ld = _round8(cols)
    m = min(rows, cols)
    ldm = _round8(m)
    x = torch.empty((2, batch, rows, ld), dtype=torch.bfloat16, device=device)
    a = torch.empty((batch, m, ldm), dtype=torch.bfloat16, device=device)
    b = torch.empty((batch, m, ldm), dtype=torch.bfloat16, device=device)
    return NSBuffers(rows, cols, batch, ld, ldm, x, a, b)


def _gemm(a, lda, abs_, a_mn, b, ldb, bbs, b_mn, d, ldd, dbs, e, epi, c1, c2, m, n, k, batch,
          status, stream, symmetric: int = 0, sums=None, scales=None, flags=None) -> None:
    _lib.launch("muzo_ns_gemm", a, lda, abs_, a_mn, b, ldb, bbs, b_mn, d, ldd, dbs, e, epi, float(c1), float(c2),
                m, n, k, batch, symmetric, sums, scales, flags, status, stream)


def ns_iterations(buf: NSBuffers, batch: int, steps: int, start_parity: int, status_ptr: int,
                  stream: int, symmetric: int = 1, sums_ptr: int | None = None, scales_ptr: int | None = None,
                  flags_ptr: int | None = None) -> int:
    """Run ``steps`` quintic iterations on the first ``batch`` matrices; return the parity of the
    buffer that holds the result. With ``sums_ptr`` (and ``scales_ptr``, ``flags_ptr``) the last
    iteration's update GEMM also accumulates each matrix's sum of (result * scale)^2 into its
    MUZO_SUM_U2 slot and flags a non-finite result (what muzo_update_sumsq does in a pass of
    its own)."""

    a_c, b_c, c_c = (np.float32(v) for v in NS_COEFFS)
    rows, cols, ld, ldm = buf.rows, buf.cols, buf.ld, buf.ldm
    m = min(rows, cols)
    x_bs = rows * ld
    m_bs = m * ldm
    pa = buf.a.data_ptr()
    pb = buf.b.data_ptr()
    tall = rows > cols
    parity = start_parity
    for it in range(int(steps)):
        last = it + 1 == int(steps)
        sums = (sums_ptr, scales_ptr, flags_ptr) if last and sums_ptr else (None, None, None)
        px = buf.x_slot(parity).data_ptr()
        py = buf.x_slot(parity ^ 1).data_ptr()
        # A = X X^T and B = b A + c A A are symmetric: only their upper-triangle tiles are
        # computed and mirrored
        if not tall:
            # A = X X^T: both operands are X's rows (K = cols contiguous)
            _gemm(px, ld, x_bs, 0, px, ld, x_bs, 0, pa, ldm, m_bs, None, _lib.EPI_STORE, 0.0, 0.0,
                  m, m, cols, batch, status_ptr, stream, symmetric)
        else:
            # X = G^T: A = G^T G reads G with M and N contiguous (MN-major), K = rows
            _gemm(px, ld, x_bs, 1, px, ld, x_bs, 1, pa, ldm, m_bs, None, _lib.EPI_STORE, 0.0, 0.0,
                  m, m, rows, batch, status_ptr, stream, symmetric)
        # B = b A + c (A @ A): second operand A[k][n] is N-contiguous (MN-major)
        _gemm(pa, ldm, m_bs, 0, pa, ldm, m_bs, 1, pb, ldm, m_bs, pa, _lib.EPI_POLY, b_c, c_c,
              m, m, m, batch, status_ptr, stream, symmetric)
        if not tall:
            # X' = a X + B @ X: X[k][n] is N-contiguous
            _gemm(pb, ldm, m_bs, 0, px, ld, x_bs, 1, py, ld, x_bs, px, _lib.EPI_UPDATE, a_c, 0.0,
                  m, cols, m, batch, status_ptr, stream, 0, *sums)
        else:
            # G' = (a X + B X)^T = a G + G B^T: B's rows are K-contiguous
            _gemm(px, ld, x_bs, 0, pb, ldm, m_bs, 0, py, ld, x_bs, px, _lib.EPI_UPDATE, a_c, 0.0,
                  rows, cols, cols, batch, status_ptr, stream, 0, *sums)
        parity ^= 1
    return parity


@torch.no_grad()
def zeropower_via_newtonschulz5(G: torch.Tensor, steps: int = 5) -> torch.Tensor:
    """Approximately orthogonalise a 2-D CUDA matrix (newton_schulz.py:17-66).

    Zero or non-finite inputs, and non-finite results, return zeros. The result has G's dtype
    (float32 for integer G).
    """

    if G.ndim != 2:
        raise ValueError("zeropower_via_newtonschulz5 accepts 2D tensors only")
    if steps < 0:
        raise ValueError("steps must be non-negative")
    if G.device.type != "cuda":
        raise ValueError("muzo_clip_b200 runs Newton-Schulz on CUDA devices only")

    out_dtype = G.dtype if G.is_floating_point() else torch.float32
    src = G if G.dtype in (torch.float32, torch.bfloat16, torch.float16) else G.to(torch.float32)
    src = src.contiguous()
    rows, cols = int(src.shape[0]), int(src.shape[1])
    if src.numel() == 0:
        return torch.zeros_like(G, dtype=out_dtype)
    device = src.device
    stream = _lib.stream_ptr(device)
    buf = allocate_ns_buffers(rows, cols, 1, device)
    scratch = torch.zeros(_lib.NSUMS + 3, dtype=torch.float64, device=device)
    sums_ptr = scratch.data_ptr()
    flags = scratch[_lib.NSUMS:].view(torch.int32)  # [flag, the GEMMs' four status words, unused]
    flags_ptr = flags.data_ptr()
    status_ptr = flags_ptr + 4

    x0 = buf.x_slot(0)[0]
    dense = buf.ld == cols
    target = x0 if dense else torch.empty((rows, cols), dtype=torch.bfloat16, device=device)
    segs, total = _lib.plan_linear([src.numel()], [src.data_ptr()], [target.data_ptr()])
    table = _lib.to_device_table(segs, device)
    _lib.launch("muzo_ns_prepare", table.data_ptr(), len(segs), total, _lib.dtype_code(src.dtype),
                                        sums_ptr, flags_ptr, stream)
    nseg, ntot = _lib.plan_linear([src.numel()], [target.data_ptr()], [target.data_ptr()])
    ntable = _lib.to_device_table(nseg, device)
    _lib.launch("muzo_ns_normalize", ntable.data_ptr(), len(nseg), ntot, sums_ptr, flags_ptr,
                                          stream)
    if not dense:
        x0[:, :cols].copy_(target)
    parity = ns_iterations(buf, 1, steps, 0, status_ptr, stream)
    result = buf.x_slot(parity)[0][:, :cols]
    flag, status = (int(v) for v in flags[:2].cpu())
    if status != 0:
        raise _lib.MuzoError(f"Newton-Schulz GEMM reported status {status}")
    if flag & (_lib.FLAG_NONFINITE_INPUT | _lib.FLAG_ZERO_NORM):
        logger.warning("Newton-Schulz input is non-finite or has zero norm; returning zeros")
        return torch.zeros_like(G, dtype=out_dtype)
    if not bool(torch.isfinite(result).all()):
        logger.warning("Newton-Schulz produced non-finite output; returning zeros")
        return torch.zeros_like(G, dtype=out_dtype)
    return result.to(dtype=out_dtype)
