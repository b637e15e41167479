"""Host-side logic of MuZOClipOptimizer against the reference package, without a GPU.

The device engine is replaced by a recording fake (test double); the reference runs on CPU
tensors. With the same scripted losses both must produce identical seeds, projections, skip
decisions, EMAs, learning-rate backoff, history and step guards (muzo_optimizer.py:190-371).
"""

from __future__ import annotations

import math
import sys

import pytest
import torch

from conftest import ROOT

from reference_pkg import reference_path

REF_PATH = reference_path()
REF = str(REF_PATH) if REF_PATH is not None else ""


def _have_reference() -> bool:
    return REF_PATH is not None


class FakeEngine:
    def __init__(self, opt, *a, **k):
        self.opt = opt
        self.calls = []
        self.blocks = [s for s in opt.selected_params]
        self.device = torch.device("cpu")

    def matches(self, opt):
        return True

    def perturb(self, seed, alpha):
        self.calls.append(("perturb", seed, alpha))

    def run_step(self, history, lr):
        self.calls.append(("step", len(history), lr))
        return {i: {"update_rms": 1e-6 * (i + 1), "ratio": 1e-3 * (i + 1)} for i in range(len(self.blocks))}


def _model():
    torch.manual_seed(0)
    m = torch.nn.Module()
    m.layers = torch.nn.ModuleList()
    for _ in range(2):
        blk = torch.nn.Module()
        blk.q_proj = torch.nn.Linear(16, 16, bias=False)
        blk.k_proj = torch.nn.Linear(16, 8, bias=False)
        blk.norm = torch.nn.LayerNorm(16)
        m.layers.append(blk)
    m.lm_head = torch.nn.Linear(16, 4, bias=False)
    return m


LOSSES = [(2.0, 2.1), (2.05, 1.95), (float("nan"), 2.0), (2.0, 2.02), (9.0, 2.0), (1.99, 2.01), (2.0, 2.0),
          (1.9, 2.0), (2.1, 1.9), (float("inf"), 1.0), (2.0, 1.98), (1.97, 2.0), (2.0, 2.03), (2.01, 2.0)]


def _closure(seq):
    it = iter(x for pair in seq for x in pair)
    return lambda: next(it)


@pytest.mark.skipif(not _have_reference(), reason="reference package not available (MUZO_REFERENCE_PATH / baseline/_ref)")
def test_projection_and_step_logic_match_reference(monkeypatch):
    sys.path.insert(0, REF)
    from muzo_clip import MuZOClipOptimizer as RefOpt

    import muzo_clip_b200.muzo_optimizer as mo

    monkeypatch.setattr(mo, "StepEngine", FakeEngine)
    kw = dict(lr=1e-3, seed=77, horizon=6, min_history=3, loss_spike_ratio=2.0)
    ref = RefOpt(_model(), **kw)
    mine = mo.MuZOClipOptimizer(_model(), **kw)
    assert mine.selected_parameter_names() == ref.selected_parameter_names()
    c_ref, c_mine = _closure(LOSSES), _closure(LOSSES)
    for _ in LOSSES:
        a = ref.estimate_projection(c_ref)
        b = mine.estimate_projection(c_mine)
        for key in a:
            va, vb = a[key], b[key]
            if isinstance(va, float) and math.isnan(va):
                assert math.isnan(vb)
            else:
                assert va == vb, (key, va, vb)
        sa = ref.step()
        sb = mine.step()
        assert sa["skipped"] == sb["skipped"] and sa["skip_reason"] == sb["skip_reason"]
        assert sa["lr"] == sb["lr"]
        if not sa["skipped"]:
            assert sa["updated_param_count"] == sb["updated_param_count"]
        for attr in ("p_abs_ema", "loss_ema", "bad_step_count", "lr_scale", "_has_pending_update",
                     "_last_step_updated"):
            assert getattr(ref, attr) == getattr(mine, attr), attr
        assert [tuple(h.__dict__.values()) for h in ref.history] == [tuple(h.__dict__.values()) for h in mine.history]


def test_failed_closure_restores_perturbation(monkeypatch):
    import muzo_clip_b200.muzo_optimizer as mo

    monkeypatch.setattr(mo, "StepEngine", FakeEngine)
    opt = mo.MuZOClipOptimizer(_model(), seed=5)
    calls = {"n": 0}

    def closure():
        calls["n"] += 1
        if calls["n"] == 2:
            raise RuntimeError("forward failed")
        return 1.0

    with pytest.raises(RuntimeError):
        opt.estimate_projection(closure)
    ev = opt._engine.calls
    # +eps, then -2eps, the failure at displacement -1 restores with +eps (muzo_optimizer.py:499-502)
    assert [c[2] for c in ev] == [pytest.approx(1e-3), pytest.approx(-2e-3), pytest.approx(1e-3)]
    assert len({c[1] for c in ev}) == 1
    assert not opt.history


def test_validation_errors_match_reference_messages():
    import muzo_clip_b200.muzo_optimizer as mo

    cases = [dict(horizon=0), dict(min_history=0), dict(min_history=9, horizon=8), dict(zo_eps=0.0),
             dict(update_ratio_clip=0.0), dict(muon_scale=0.0), dict(distribution="uniform")]
    msgs = ["horizon must be positive", "min_history must be positive",
            "min_history must be less than or equal to horizon", "zo_eps must be positive",
            "update_ratio_clip must be positive", "muon_scale must be positive", "Unsupported distribution: uniform"]
    for kw, msg in zip(cases, msgs):
        with pytest.raises(ValueError, match=msg):
            mo.MuZOClipOptimizer(_model(), **kw)


def test_cpu_tensors_are_rejected_not_computed():
    from muzo_clip_b200 import make_zo_noise_like, zeropower_via_newtonschulz5

    with pytest.raises(ValueError):
        make_zo_noise_like(torch.zeros(4, 4), 1, "w")
    with pytest.raises(ValueError):
        zeropower_via_newtonschulz5(torch.ones(4, 4))
    with pytest.raises(TypeError):
        make_zo_noise_like(torch.zeros(4, 4, dtype=torch.int32), 1, "w")


def test_state_dict_resumes_identically(monkeypatch):
    """Resume format (the reference keeps this state only in memory): a restored optimizer
    continues with the same seeds, projections and statistics as the uninterrupted one."""
    import json

    import muzo_clip_b200.muzo_optimizer as mo

    monkeypatch.setattr(mo, "StepEngine", FakeEngine)
    kw = dict(lr=1e-3, seed=21, horizon=5, min_history=2)
    a = mo.MuZOClipOptimizer(_model(), **kw)
    closure = _closure(LOSSES)
    for _ in range(5):
        a.estimate_projection(closure)
        a.step()
    saved = json.loads(json.dumps(a.state_dict()))  # must survive a JSON round trip
    b = mo.MuZOClipOptimizer(_model(), **kw)
    b.load_state_dict(saved)
    rest = LOSSES[5:]
    ca, cb = _closure(rest), _closure(rest)
    for _ in rest:
        pa, pb = a.estimate_projection(ca), b.estimate_projection(cb)
        assert {k: v for k, v in pa.items() if not (isinstance(v, float) and math.isnan(v))} == \
            {k: v for k, v in pb.items() if not (isinstance(v, float) and math.isnan(v))}
        assert a.step() == b.step()
    with pytest.raises(ValueError):
        c = mo.MuZOClipOptimizer(torch.nn.Linear(4, 4), **kw)
        c.load_state_dict(saved)


def _public_members(module):
    import inspect

    return {n: o for n, o in vars(module).items()
            if not n.startswith("_") and (inspect.isfunction(o) or inspect.isclass(o))
            and getattr(o, "__module__", None) == module.__name__}


def _assert_compatible(ref_fn, mine_fn, where: str) -> None:
    """Every parameter of the reference callable exists here with the same kind and default;
    parameters added here have defaults."""
    import inspect

    ref_sig, mine_sig = inspect.signature(ref_fn), inspect.signature(mine_fn)
    for name, p in ref_sig.parameters.items():
        assert name in mine_sig.parameters, f"{where}: parameter {name} missing"
        q = mine_sig.parameters[name]
        assert q.kind == p.kind, f"{where}: {name} is {q.kind}, reference {p.kind}"
        assert q.default == p.default, f"{where}: default of {name}"
    for name, q in mine_sig.parameters.items():
        if name not in ref_sig.parameters:
            assert q.default is not inspect.Parameter.empty or q.kind in (q.VAR_KEYWORD, q.VAR_POSITIONAL), \
                f"{where}: added parameter {name} needs a default"


@pytest.mark.skipif(not _have_reference(), reason="reference package not available (MUZO_REFERENCE_PATH / baseline/_ref)")
def test_public_api_matches_reference():
    """The drop-in contract: every public function, class, method, property and dataclass field
    of the reference's modules exists here with compatible parameters and the same defaults."""
    import dataclasses
    import importlib
    import inspect

    sys.path.insert(0, REF)
    try:
        ref_pkg = importlib.import_module("muzo_clip")
        mine_pkg = importlib.import_module("muzo_clip_b200")
        assert set(ref_pkg.__all__) <= set(mine_pkg.__all__)
        checked = 0
        for mod in ("muzo_optimizer", "newton_schulz", "parameter_filter", "prng", "qk_clip", "integration"):
            ref_mod = importlib.import_module(f"muzo_clip.{mod}")
            mine_mod = importlib.import_module(f"muzo_clip_b200.{mod}")
            for name, ref_obj in _public_members(ref_mod).items():
                mine_obj = getattr(mine_mod, name, None)
                assert mine_obj is not None, f"{mod}.{name} missing"
                if inspect.isfunction(ref_obj):
                    _assert_compatible(ref_obj, mine_obj, f"{mod}.{name}")
                    checked += 1
                    continue
                if dataclasses.is_dataclass(ref_obj):
                    assert [f.name for f in dataclasses.fields(ref_obj)] == \
                        [f.name for f in dataclasses.fields(mine_obj)], f"{mod}.{name} fields"
                    checked += 1
                    continue
                _assert_compatible(ref_obj.__init__, mine_obj.__init__, f"{mod}.{name}.__init__")
                for attr, member in vars(ref_obj).items():
                    if attr.startswith("_"):
                        continue
                    mine_member = inspect.getattr_static(mine_obj, attr, None)
                    assert mine_member is not None, f"{mod}.{name}.{attr} missing"
                    if isinstance(member, property):
                        assert isinstance(mine_member, property), f"{mod}.{name}.{attr} is not a property"
                    elif inspect.isfunction(member):
                        _assert_compatible(member, getattr(mine_obj, attr), f"{mod}.{name}.{attr}")
                    checked += 1
        assert checked >= 25  # the loops above did run over the whole surface
    finally:
        if REF in sys.path:
            sys.path.remove(REF)


@pytest.mark.parametrize("rows, cols, batch", [(4096, 14336, 3), (14336, 4096, 2), (1000, 1003, 4), (7, 9, 1),
                                               (256, 256, 16)])
def test_newton_schulz_workspace_layout(rows, cols, batch):
    """The workspace carved from one flat buffer of ns_workspace_bytes: iterate X [2, batch,
    rows, ld] and A, B [batch, m, ldm] fit, do not overlap, keep 16-byte aligned rows (ld, ldm
    multiples of 8) and 256-byte aligned bases; a buffer that cannot hold them is refused."""
    from muzo_clip_b200.newton_schulz import ns_buffers_in, ns_workspace_bytes

    nbytes = ns_workspace_bytes(rows, cols, batch)
    raw = torch.empty(nbytes, dtype=torch.uint8)
    buf = ns_buffers_in(raw, rows, cols, batch)
    m = min(rows, cols)
    assert buf.ld % 8 == 0 and buf.ld >= cols and buf.ldm % 8 == 0 and buf.ldm >= m
    assert tuple(buf.x.shape) == (2, batch, rows, buf.ld)
    assert tuple(buf.a.shape) == tuple(buf.b.shape) == (batch, m, buf.ldm)
    base = raw.data_ptr()
    spans = sorted((t.data_ptr() - base, t.data_ptr() - base + t.numel() * t.element_size())
                   for t in (buf.x, buf.a, buf.b))
    assert spans[0][0] == 0 and spans[-1][1] <= nbytes
    assert all(lo % 256 == 0 for lo, _ in spans)
    assert all(spans[i][1] <= spans[i + 1][0] for i in range(len(spans) - 1))
    with pytest.raises(ValueError):  # one byte short of the last view
        ns_buffers_in(raw[: spans[-1][1] - 1], rows, cols, batch)
