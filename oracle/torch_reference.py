"""The reference's PyTorch path for the optimizer hot path, restated op for op — TEST AND BENCHMARK
INFRASTRUCTURE (the oracle of the torch-level behaviour; the product never imports it).

turfur44/MuZO-Clip computes everything with PyTorch ops; on a B200 those ops *are* the reference
behaviour (torch's CUDA Philox generator, element-wise kernels, cuBLAS bf16 GEMMs). The reference
package cannot be assumed importable where the GPU tests run, so this module repeats its
tensor-op sequence (same ops, same order, same dtypes) for the parity tests, the golden-vector
generator and the CPU baseline of bench.py. tests/test_reference_link_cpu.py (CPU tensors) and
tests/test_reference_link_gpu.py (CUDA tensors, the bf16 Newton-Schulz branch) prove it equal to
the real package, bit for bit, wherever that package can be imported.

Line references are to the reference's muzo_clip/ package.
"""

from __future__ import annotations

import hashlib
import math

import torch


def hash64_seed(base_seed, param_name, param_shape, block_index=0) -> int:
    """prng.py:19-36."""
    text = "|".join([str(int(base_seed)), param_name, ",".join(str(int(d)) for d in param_shape),
                     str(int(block_index))])
    digest = hashlib.blake2b(text.encode("utf-8"), digest_size=8).digest()
    return int.from_bytes(digest, "little") & ((1 << 63) - 1)


def noise_like(tensor: torch.Tensor, base_seed: int, name: str, block_index: int = 0,
               distribution: str = "normal") -> torch.Tensor:
    """prng.py:59-81: fresh generator on the tensor's device, fp32 randn or int8 randint{0,1}
    mapped to +-1, cast to the tensor's dtype."""
    key = hash64_seed(int(base_seed), name, tuple(tensor.shape), int(block_index))
    gen = torch.Generator(device=tensor.device)
    gen.manual_seed(key)
    if distribution == "normal":
        z = torch.randn(tensor.shape, generator=gen, device=tensor.device, dtype=torch.float32)
    else:
        z = torch.randint(low=0, high=2, size=tensor.shape, generator=gen, device=tensor.device,
                          dtype=torch.int8).to(torch.float32)
        z.mul_(2.0).sub_(1.0)
    return z.to(dtype=tensor.dtype)


def param_blocks(param: torch.Tensor, block_rows):
    """prng.py:84-106."""
    if block_rows is None:
        return [(0, param)]
    out = []
    for bi, start in enumerate(range(0, int(param.shape[0]), int(block_rows))):
        out.append((bi, param[start:min(start + int(block_rows), int(param.shape[0]))]))
    return out


@torch.no_grad()
def perturb(named_params, seed: int, scaling_factor: float, zo_eps: float, distribution: str,
            block_rows=None) -> None:
    """muzo_optimizer.py:434-446."""
    scale = float(scaling_factor) * zo_eps
    for name, p in named_params:
        for bi, block in param_blocks(p.data, block_rows):
            block.add_(noise_like(block, seed, name, bi, distribution), alpha=scale)


@torch.no_grad()
def rebuild(block: torch.Tensor, name: str, block_index: int, history, beta: float,
            distribution: str, normalize: bool) -> torch.Tensor:
    """muzo_optimizer.py:318-333; history items have .seed and .p, oldest first."""
    M = torch.zeros(block.shape, device=block.device, dtype=torch.float32)
    coeff_sum = 0.0
    for age, item in enumerate(reversed(history)):
        coeff = beta ** age
        z = noise_like(block, item.seed, name, block_index, distribution).float()
        M.add_(z, alpha=coeff * item.p)
        coeff_sum += coeff
    if normalize and coeff_sum > 0:
        M.div_(coeff_sum)
    return M


@torch.no_grad()
def newton_schulz(G: torch.Tensor, steps: int = 5) -> torch.Tensor:
    """newton_schulz.py:17-66 (bf16 on CUDA, fp32 on CPU)."""
    out_dtype = G.dtype if G.is_floating_point() else torch.float32
    zeros = torch.zeros_like(G, dtype=out_dtype)
    if not bool(torch.isfinite(G).all().item()):
        return zeros
    norm = G.float().norm()
    if not bool(torch.isfinite(norm).item()) or float(norm.item()) <= 0.0:
        return zeros
    a, b, c = (3.4445, -4.7750, 2.0315)
    X = G.to(dtype=torch.bfloat16 if G.device.type == "cuda" else torch.float32)
    transposed = G.size(0) > G.size(1)
    if transposed:
        X = X.mT
    X = X / (X.float().norm() + 1e-7)
    for _ in range(int(steps)):
        A = X @ X.mT
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    if transposed:
        X = X.mT
    if not bool(torch.isfinite(X).all().item()):
        return zeros
    return X.to(dtype=out_dtype)


def _rms(t: torch.Tensor) -> torch.Tensor:
    return t.float().pow(2).mean().sqrt()


@torch.no_grad()
def apply_update(block: torch.Tensor, U: torch.Tensor, lr: float, muon_scale: float,
                 ratio_clip: float, weight_decay: float):
    """muzo_optimizer.py:340-357 for one block; returns (update_rms, ratio)."""
    U.mul_(math.sqrt(max(int(block.shape[0]), int(block.shape[1]))) * muon_scale)
    update_rms = _rms(U) * lr
    weight_rms = _rms(block)
    ratio = float((update_rms / (weight_rms + 1e-12)).item())
    if ratio > ratio_clip:
        U.mul_(ratio_clip / ratio)
        update_rms = _rms(U) * lr
        ratio = float((update_rms / (weight_rms + 1e-12)).item())
    block.add_(U.to(dtype=block.dtype), alpha=-lr)
    if weight_decay:
        block.mul_(1.0 - lr * weight_decay)
    return float(update_rms.item()), ratio


@torch.no_grad()
def step(named_params, history, *, lr, beta, ns_steps, muon_scale, ratio_clip, weight_decay,
         distribution, normalize=True, block_rows=None):
    """The body of step() (muzo_optimizer.py:310-371) for a non-empty history."""
    rms_values, ratio_max, count = [], 0.0, 0
    for name, p in named_params:
        for bi, block in param_blocks(p.data, block_rows):
            M = rebuild(block, name, bi, history, beta, distribution, normalize)
            U = newton_schulz(M, steps=ns_steps)
            if not bool(torch.isfinite(U.float()).all().item()):
                continue
            urms, ratio = apply_update(block, U, lr, muon_scale, ratio_clip, weight_decay)
            rms_values.append(urms)
            ratio_max = max(ratio_max, ratio)
            count += 1
    mean = sum(rms_values) / len(rms_values) if rms_values else 0.0
    return {"update_rms_mean": mean, "update_ratio_max": ratio_max, "updated_param_count": count}


def qk_head_max(logits: torch.Tensor) -> torch.Tensor:
    """qk_clip.py:194."""
    return logits.float().amax(dim=(0, 2, 3)).cpu()


def eager_logits(q: torch.Tensor, k: torch.Tensor, scaling: float, causal: bool) -> torch.Tensor:
    """Pre-softmax logits of transformers' eager attention: repeat_kv, matmul * scaling, plus the
    causal mask at the dtype's minimum."""
    group = q.shape[1] // k.shape[1]
    kr = k[:, :, None].expand(k.shape[0], k.shape[1], group, k.shape[2], k.shape[3]).reshape(
        k.shape[0], k.shape[1] * group, k.shape[2], k.shape[3])
    w = torch.matmul(q, kr.transpose(2, 3)) * scaling
    if causal:
        sq, sk = q.shape[2], k.shape[2]
        i = torch.arange(sq, device=q.device)[:, None] + (sk - sq)
        j = torch.arange(sk, device=q.device)[None, :]
        mask = torch.zeros((sq, sk), dtype=w.dtype, device=q.device)
        mask.masked_fill_(j > i, torch.finfo(w.dtype).min)
        w = w + mask
    return w


@torch.no_grad()
def qk_scale(q_weight: torch.Tensor, k_weight: torch.Tensor, smax: torch.Tensor, tau: float, alpha: float):
    """qk_clip.py:235-310 for one module with per-head maxima ``smax`` (CPU fp32)."""
    needs_clip = smax > tau
    if not bool(needs_clip.any().item()):
        return 0, False
    gamma = torch.clamp(tau / smax.clamp_min(1e-12), max=1.0)
    hq = int(gamma.numel())
    hd = q_weight.shape[0] // hq
    hk = k_weight.shape[0] // hd
    gamma = gamma.to(device=q_weight.device, dtype=torch.float32)
    needs_clip = needs_clip.to(device=q_weight.device)
    q_scale = gamma.pow(alpha).to(dtype=q_weight.dtype)
    for h in range(hq):
        if bool(needs_clip[h].item()):
            q_weight[h * hd:(h + 1) * hd].mul_(q_scale[h])
    group = hq // hk
    ks, km = [], []
    for g in range(hk):
        ks.append(gamma[g * group:(g + 1) * group].min())
        km.append(bool(needs_clip[g * group:(g + 1) * group].any().item()))
    kst = torch.stack(ks).pow(1.0 - alpha).to(dtype=k_weight.dtype)
    nk = 0
    for g, m in enumerate(km):
        if m:
            k_weight[g * hd:(g + 1) * hd].mul_(kst[g])
            nk += 1
    return int(needs_clip.sum().item()) + nk, False
