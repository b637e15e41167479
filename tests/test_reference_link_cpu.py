"""The restatement of the reference's op sequence (oracle/torch_reference.py), which the
GPU parity tests and the golden vectors build on, against the real reference package on CPU
tensors, bit for bit; and the committed hash known answers against the package itself.

Skips when the reference package cannot be imported (MUZO_REFERENCE_PATH, or the offline install
under baseline/_ref). On CPU, the reference's Newton-Schulz takes its fp32 branch
(muzo_clip/newton_schulz.py:46); tests/test_reference_link_gpu.py pins the bf16 CUDA branch.
"""

from __future__ import annotations

import json

import pytest
import torch

import check_against_reference as car
from conftest import GOLDEN
from reference_pkg import import_reference

ref = import_reference()
pytestmark = pytest.mark.skipif(ref is None, reason="reference package not available (MUZO_REFERENCE_PATH / baseline/_ref)")

CPU = torch.device("cpu")


def test_hash_known_answers_are_the_reference_outputs():
    import muzo_clip.prng  # noqa: F401

    kat = car.hash_kat(ref)
    assert kat == json.loads((GOLDEN / "hash_kat.json").read_text())


def test_noise_restatement_matches_reference():
    import muzo_clip.prng  # noqa: F401

    car.check_noise(ref, CPU)


def test_newton_schulz_restatement_matches_reference():
    import muzo_clip.newton_schulz  # noqa: F401

    car.check_newton_schulz(ref, CPU)


def test_step_and_perturb_restatement_match_reference_optimizer():
    car.check_step_and_perturb(ref, CPU)
