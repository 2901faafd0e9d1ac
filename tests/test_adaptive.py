"""The online per-layer allocator (AdaptiveLayerController) and its exact
knapsack, against decision logs of the reference's own controller
(tests/golden/adaptive.json, written by tests/golden/make_golden.py from the
reference's adaptive.py:68-335 driven by its simulated per-layer environment,
sim.py:131-167).

A seeded controller fed the accepted counts the reference's environment
returned must choose the same plan and gamma in every round; the reference's
own test properties (the sensitive layer found, the byte budget never
exceeded, the probe rate bounded, the throttle) are checked on the replays.
"""

import json

import numpy as np
import pytest

from draftkv import CompressionConfig, CostModel, LayerPlan
from draftkv.adaptive import AdaptiveLayerController
from draftkv.layers import SensitivityProfile, allocate
from tests.golden import make_golden as G


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.loads((golden_dir / "adaptive.json").read_text())


class _Pkg:
    CompressionConfig = CompressionConfig
    CostModel = CostModel
    LayerPlan = LayerPlan


def _replay(name, golden):
    """Runs our controller through the recorded scenario; returns it, the
    candidates, the budget and the plans it chose."""
    _, kw, phases = next(s for s in G.ADAPTIVE_SCENARIOS if s[0] == name)
    cands, cm, budget = G.adaptive_setup(_Pkg)
    kw = dict(kw)
    b = budget(kw.pop("budget"))
    ctrl = AdaptiveLayerController(cm, G.ADAPTIVE_NL, b, cands, ctx_hint=G.ADAPTIVE_CTX, **kw)
    rec = golden["logs"][name]["rounds"]
    keys = [key for _d, _s, n, key in phases for _ in range(n)]
    plans = []
    for rd, ((want_plan, want_g, k), key) in enumerate(zip(rec, keys)):
        plan, g = ctrl.select(G.ADAPTIVE_CTX, key)
        assert [cands.index(c) for c in plan] == want_plan and g == want_g, (name, rd)
        ctrl.update(plan, g, k, G.ADAPTIVE_CTX, key)
        plans.append(plan)
    return ctrl, cands, b, plans


@pytest.mark.parametrize("name", [s[0] for s in G.ADAPTIVE_SCENARIOS])
def test_decisions_match_the_reference(golden, name):
    ctrl, _, _, _ = _replay(name, golden)
    want = golden["logs"][name]
    assert ctrl.n_probes == want["probes"]
    assert ctrl.n_resolves == want["resolves"]
    assert ctrl.n_stall_recoveries == want["recoveries"]
    for key, d in want["damages"].items():
        np.testing.assert_allclose(ctrl.damages(None if key == "None" else key), d, rtol=0, atol=1e-12)


def test_finds_the_sensitive_layer(golden):
    """Reference tests/test_adaptive.py:47-56: the layer with the damage
    is found and protected by the plan."""
    ctrl, cands, _, _ = _replay("find", golden)
    assert int(np.argmax(ctrl.damages())) == 2
    plan = ctrl.plans[None]
    assert cands.index(plan[2]) >= max(cands.index(plan[L]) for L in range(G.ADAPTIVE_NL) if L != 2)


def test_tracks_a_shift_and_keys_hold_their_own_plans(golden):
    """Reference tests/test_adaptive.py:73-95."""
    ctrl, _, _, _ = _replay("shift", golden)
    assert int(np.argmax(ctrl.damages())) == 4
    ctrl, _, _, _ = _replay("keys", golden)
    assert int(np.argmax(ctrl.damages("prose"))) == 0
    assert int(np.argmax(ctrl.damages("code"))) == 5


@pytest.mark.parametrize("name", ["find", "rate", "stall"])
def test_never_exceeds_the_byte_budget(golden, name):
    """Reference tests/test_adaptive.py:59-70: probes may spend less, never more."""
    _, _, b, plans = _replay(name, golden)
    for p in plans:
        assert p.per_layer_bytes(G.ADAPTIVE_CTX, 12, 64) <= b + 1e-6


def test_probe_rate_and_throttle(golden):
    """Reference tests/test_adaptive.py:98-125."""
    ctrl, _, _, _ = _replay("rate", golden)
    assert 0.02 <= ctrl.n_probes / ctrl.n_decisions <= 0.18
    for resync, want in golden["probe"].items():
        cands, cm, budget = G.adaptive_setup(_Pkg, float(resync))
        c = AdaptiveLayerController(cm, G.ADAPTIVE_NL, budget(0.6), cands, ctx_hint=G.ADAPTIVE_CTX,
                                    probe_prob=0.3, seed=1)
        assert [c.effective_probe_prob(x) for x in (256, 4096, G.ADAPTIVE_CTX)] == want
    assert golden["probe"]["1e-08"][2] == pytest.approx(0.3)
    assert golden["probe"]["2e-06"][2] < 0.05


def test_exact_knapsack_matches_the_reference(golden):
    cands, _, budget = G.adaptive_setup(_Pkg)
    for case in golden["knapsack"]:
        prof = SensitivityProfile(cands[-1], 0.9, tuple(cands))
        for L, ci, a in case["alpha"]:
            prof.alpha[(L, cands[ci])] = a
        plan = allocate(prof, budget(case["frac"]), G.ADAPTIVE_CTX, 12, 64, G.ADAPTIVE_NL)
        assert [cands.index(c) for c in plan] == case["plan"]


def test_rebuild_cost_uses_the_measured_rebuild_rate():
    """A cost model calibrated on the device carries its own per-position
    rebuild cost; the probe throttle reads it through rebuild_cost."""
    cands, cm, budget = G.adaptive_setup(_Pkg, 1.0e-8)
    from dataclasses import replace
    slow = replace(cm, rebuild_per_token=2.0e-6)
    assert slow.rebuild_cost(32768, 2) == pytest.approx(32768 * 2.0e-6 * 2 / G.ADAPTIVE_NL)
    fast = AdaptiveLayerController(cm, G.ADAPTIVE_NL, budget(0.6), cands, ctx_hint=G.ADAPTIVE_CTX, probe_prob=0.3)
    dear = AdaptiveLayerController(slow, G.ADAPTIVE_NL, budget(0.6), cands, ctx_hint=G.ADAPTIVE_CTX, probe_prob=0.3)
    assert fast.effective_probe_prob(G.ADAPTIVE_CTX) == pytest.approx(0.3)
    assert dear.effective_probe_prob(G.ADAPTIVE_CTX) < 0.05
