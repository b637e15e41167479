"""The CPU oracle against the golden vectors torch produced on a B200 (tests/golden/*.npz).

This pins the oracle: the Philox counter layout and torch's launch split (Rademacher noise must
match bit for bit, including tensors torch splits into several launches), the Box-Muller pairing
of normal noise (to 1e-5 relative / 2e-6 absolute), the fp32 fused multiply-add of the
perturbation and rebuild, the reciprocal-multiply normalisation of the momentum, and the update
arithmetic. No GPU is needed.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN

import muzo_oracle as orc

NOISE = np.load(GOLDEN / "noise_cuda.npz")
STEP = np.load(GOLDEN / "step_cuda.npz")


def _noise_cases():
    names = sorted({k.split(".")[0] for k in NOISE.files})
    return names


@pytest.mark.parametrize("name", _noise_cases())
def test_noise_matches_golden(name):
    key = int(NOISE[f"{name}.key"][0])
    numel = int(NOISE[f"{name}.numel"][0])
    dist = "rademacher" if name.startswith("r") else "normal"
    if f"{name}.bits" in NOISE.files:
        z = orc.noise(numel, key, dist)
        bits = np.unpackbits(NOISE[f"{name}.bits"])[:numel]
        assert np.array_equal((z > 0).astype(np.uint8), bits)
        return
    idx = NOISE[f"{name}.idx"]
    val = NOISE[f"{name}.val"]
    z = orc.noise(numel, key, dist, indices=idx)
    if dist == "rademacher":
        # stored as torch's randint{0,1} words; the reference maps them to 2b - 1
        assert np.array_equal(z, val.astype(np.float32) * 2 - 1)
    else:
        np.testing.assert_allclose(z, val, rtol=1e-5, atol=2e-6)


def test_split_launch_offsets_are_pinned():
    """The split cases differ from a single launch: using the unsplit layout must fail."""
    name = "r_split"
    key = int(NOISE[f"{name}.key"][0])
    numel = int(NOISE[f"{name}.numel"][0])
    idx = NOISE[f"{name}.idx"]
    val = NOISE[f"{name}.val"].astype(np.float32) * 2 - 1
    hi = idx >= numel // 2
    wrong = orc.noise(numel, key, "rademacher", indices=idx[hi], sm_count=148, max_threads=2048)
    assert np.array_equal(wrong, val[hi])
    # a planted mistake: forgetting the whole-tensor charge shifts the second half's stream
    launches = orc.noise_launches(numel, 1)
    assert len(launches) == 2 and launches[1].offset != launches[0].offset


def _bf16_ulp(x):
    ax = np.maximum(np.abs(x.astype(np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(ax)) - 7)


@pytest.mark.parametrize("dist", ["normal", "rademacher"])
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_perturb_matches_golden(dist, dt):
    w0 = STEP[f"perturb.{dist}.{dt}.in"]
    out = STEP[f"perturb.{dist}.{dt}.out"]
    key = orc.hash64_seed(77, "golden.perturb.weight", w0.shape, 0)
    mine = orc.perturb(w0, key, 1e-3, dist, dt)
    if dist == "rademacher":
        assert np.array_equal(mine, out)
    elif dt == "f32":
        # the weight's own fp32 ulp (~4e-9 at |w| ~ 0.03) bounds the difference of tiny updates
        np.testing.assert_allclose(mine - w0, out - w0, rtol=1e-5, atol=1e-8)
    else:
        # a normal value within ~1e-6 of a bf16 rounding boundary may round the other way, moving
        # alpha * z by alpha * ulp(z) (|z| < 8)
        assert np.all(np.abs(mine - out) <= _bf16_ulp(out) + 1e-3 * 8 * 2.0 ** -7)
        assert np.mean(mine == out) > 0.999


@pytest.mark.parametrize("dist", ["normal", "rademacher"])
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_rebuild_matches_golden(dist, dt):
    M_ref = STEP[f"rebuild.{dist}.{dt}.M"]
    seeds = STEP["hist.seed"]
    ps = STEP["hist.p"]
    keys, alphas = [], []
    coeff_sum = 0.0
    for age, (seed, p) in enumerate(zip(seeds[::-1], ps[::-1])):
        c = 0.9 ** age
        keys.append(orc.hash64_seed(int(seed), "golden.rebuild.weight", M_ref.shape, 0))
        alphas.append(float(np.float32(c * p)))
        coeff_sum += c
    inv = float(np.float32(1.0) / np.float32(coeff_sum))
    M = orc.rebuild(M_ref.shape, keys, alphas, dist, dt, inv)
    if dist == "rademacher":
        assert np.array_equal(M, M_ref)  # fused multiply-adds and the reciprocal multiply, bit-exact
    elif dt == "f32":
        np.testing.assert_allclose(M, M_ref, rtol=1e-5, atol=1e-6)
    else:
        # bf16 params round each z to bf16 first: a z near a rounding boundary flips by one bf16
        # ulp in rare elements (bounded by sum |alpha| * ulp); everything else to 1e-5
        close = np.isclose(M, M_ref, rtol=1e-5, atol=1e-6)
        assert np.mean(~close) < 2e-3
        bound = sum(abs(a) for a in alphas) * inv * 2.0 ** -7 * 8
        assert np.abs(M - M_ref).max() <= bound


@pytest.mark.parametrize("shape", ["64x96", "96x64", "256x688", "688x256"])
def test_newton_schulz_oracle_against_golden(shape):
    G = STEP[f"ns.{shape}.G"]
    X = STEP[f"ns.{shape}.X"]
    exact = orc.ns5_bf16(G, 5, exact=True)
    fp32 = orc.ns5_bf16(G, 5)
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))  # noqa: E731
    # the reference's cuBLAS result sits 2-4 % from the exact-accumulation iteration; the fp32
    # accumulation oracle within 1 %
    assert rel(X, exact) < 5e-2
    assert rel(fp32, exact) < 1.5e-2
    assert X.shape == G.shape


@pytest.mark.parametrize("shape", ["64x96", "96x64", "256x688", "688x256"])
def test_exact_ns_torch_matches_oracle(shape):
    """The torch float64 exact-accumulation iteration (the GPU tests' large-shape checker) is the
    numpy oracle's exact iteration: both accumulate in float64, so they may differ only where the
    two BLAS libraries' float64 sums round to different fp32 values (a handful of elements)."""
    import torch
    from exact_ns import ns5_exact

    G = STEP[f"ns.{shape}.G"]
    want = orc.ns5_bf16(G, 5, exact=True)
    got = ns5_exact(torch.from_numpy(np.ascontiguousarray(G))).numpy()
    assert got.shape == want.shape
    rel = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    assert np.mean(got == want) > 0.99 and rel < 1e-3, (np.mean(got == want), rel)
    z = np.zeros((8, 8), np.float32)
    assert not ns5_exact(torch.from_numpy(z)).any()


@pytest.mark.parametrize("tag", ["clip", "noclip"])
def test_apply_matches_golden(tag):
    w0 = STEP[f"apply.{tag}.w0"]
    U = STEP[f"apply.{tag}.U"]
    w1 = STEP[f"apply.{tag}.w1"]
    urms, ratio, lr = STEP[f"apply.{tag}.stats"]
    res = orc.apply_update(w0, U, float(lr), 0.2, 0.01, 0.01, "bf16")
    assert res.clipped == (tag == "clip")
    np.testing.assert_allclose(res.update_rms, urms, rtol=1e-5)
    np.testing.assert_allclose(res.ratio, ratio, rtol=1e-5)
    assert np.all(np.abs(res.w - w1) <= _bf16_ulp(w1))
    assert np.mean(res.w == w1) > 0.999


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_qk_max_matches_golden(dt):
    q = STEP[f"qk.{dt}.q"]
    k = STEP[f"qk.{dt}.k"]
    smax = STEP[f"qk.{dt}.smax"]
    mine = orc.qk_max(q, k, 32 ** -0.5, True, "bf16" if dt == "bf16" else "f32")
    if dt == "bf16":
        assert np.all(np.abs(mine - smax) <= _bf16_ulp(smax))
    else:
        np.testing.assert_allclose(mine, smax, rtol=1e-5)


def test_bf16_rounding_ties_to_even():
    x = np.asarray([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -1.0 - 2 ** -8, 3.0e38, np.inf], dtype=np.float32)
    r = orc.bf16_round(x)
    assert r[0] == 1.0 and r[1] == np.float32(1.0 + 2 ** -6) and r[2] == -1.0
    assert np.isinf(r[4])


def test_partition_balances_llama_layers():
    from muzo_clip_b200._engine import ns_flops, partition_blocks

    shapes = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096), (4096, 14336)]
    costs = [ns_flops(r, c, 5) for _ in range(32) for r, c in shapes]
    for world in (2, 4, 8):
        owner = partition_blocks(costs, world)
        loads = [sum(c for c, o in zip(costs, owner) if o == r) for r in range(world)]
        assert max(loads) / min(loads) < 1.02, (world, loads)
        assert partition_blocks(costs, world) == owner  # deterministic on every rank


def test_philox_published_known_answers():
    """Philox4x32-10 against the known-answer vectors published with the Random123 library
    (Salmon et al., SC'11): zero counter/key, all-ones counter/key, and the pi-digits case."""
    cases = [
        ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
        ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
        ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
         (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
    ]
    for ctr, key, want in cases:
        words = orc.philox4x32_10(*(np.array([c], np.uint64) for c in ctr), key[0] | (key[1] << 32))
        assert tuple(int(w[0]) for w in words) == want
