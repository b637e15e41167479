"""The reference package itself on a B200 (CUDA tensors): its bf16 Newton-Schulz branch
(muzo_clip/newton_schulz.py:46-58, cuBLAS), its CUDA noise and its optimizer step against the
restatement in oracle/torch_reference.py, bit for bit; the committed CUDA golden vectors
reproduced by the reference's own functions; and this build's perturbation against the reference
optimizer's, bit for bit.

Skips when the reference package cannot be imported on the machine (MUZO_REFERENCE_PATH, or the
offline install under baseline/_ref that travels with the working tree).
"""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

import check_against_reference as car
from conftest import GOLDEN
from reference_pkg import import_reference

ref = import_reference()
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(ref is None, reason="reference package not available (MUZO_REFERENCE_PATH / baseline/_ref)")]


def test_noise_restatement_matches_reference_on_cuda(device):
    import muzo_clip.prng  # noqa: F401

    car.check_noise(ref, device)


def test_bf16_newton_schulz_branch_matches_restatement(device):
    import muzo_clip.newton_schulz  # noqa: F401

    car.check_newton_schulz(ref, device)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_reference_optimizer_step_matches_restatement_on_cuda(device, dtype):
    car.check_step_and_perturb(ref, device, dtype)


def test_golden_vectors_are_the_reference_functions_outputs(device):
    """tests/golden/step_cuda.npz (perturbation, Newton-Schulz) reproduced on this B200 by the
    reference package's make_zo_noise_like and zeropower_via_newtonschulz5."""
    import muzo_clip.newton_schulz  # noqa: F401
    import muzo_clip.prng  # noqa: F401

    step = np.load(GOLDEN / "step_cuda.npz")
    for dist in ("normal", "rademacher"):
        for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            w = torch.from_numpy(step[f"perturb.{dist}.{dt_name}.in"]).to(dt).to(device)
            # the body of _perturb_selected (muzo_optimizer.py:434-446) for one block
            w.add_(ref.prng.make_zo_noise_like(w, 77, "golden.perturb.weight", 0, dist), alpha=1.0 * 1e-3)
            assert np.array_equal(w.float().cpu().numpy(), step[f"perturb.{dist}.{dt_name}.out"]), (dist, dt_name)
    for shape in ("64x96", "96x64", "256x688", "688x256"):
        G = torch.from_numpy(step[f"ns.{shape}.G"]).to(device)
        X = ref.newton_schulz.zeropower_via_newtonschulz5(G, 5).cpu().numpy()
        assert np.array_equal(X, step[f"ns.{shape}.X"]), shape


def test_perturbation_matches_reference_optimizer_bit_for_bit(device):
    """This build's projection passes against the reference optimizer's own _perturb_selected on
    a twin (bf16 tiny Llama, normal and Rademacher noise, with and without row blocks)."""
    from muzo_clip_b200 import MuZOClipOptimizer

    for dist, block_rows in (("normal", None), ("rademacher", None), ("normal", 40)):
        model = car._tiny_model(device, torch.bfloat16)
        twin = copy.deepcopy(model)
        mine = MuZOClipOptimizer(model, distribution=dist, block_rows=block_rows, seed=3)
        theirs = ref.MuZOClipOptimizer(twin, distribution=dist, block_rows=block_rows, seed=3)
        assert mine.selected_parameter_names() == theirs.selected_parameter_names()
        for seed, s in ((5, 1.0), (5, -2.0), (5, 1.0), (6, 1.0)):
            mine._perturb_selected(seed, s)
            theirs._perturb_selected(seed, s)
            for (n, p), (_, q) in zip(model.named_parameters(), twin.named_parameters()):
                assert torch.equal(p, q), (dist, block_rows, seed, s, n)
