"""The device-calibrated cost model (draftkv/calibrate.py): the constants fitted
from measured phase times, and controllers consuming them (CPU only: the
timings are given, the GPU run measures them in bench.py)."""

import pytest

from draftkv import CompressionConfig, CostModel, ThompsonController, default_arms
from draftkv.calibrate import fit_constants

CFG = CompressionConfig(8, 1.0)


def _cm():
    return CostModel(n_layers=32, n_kv_heads=8, d_head=128, weight_bytes=15.0e9, bandwidth=6.5e12, batch=4)


def test_fit_recovers_the_fixed_costs():
    cm = _cm()
    ctx, g = 32768, 2
    w = cm.weight_bytes / cm.bandwidth
    t_d = w + cm.draft_kv_bytes(CFG, ctx) / cm.bandwidth + cm.compute_per_token + 1.5e-3
    t_v = w + cm.full_kv_bytes(ctx) / cm.bandwidth + (g + 1) * cm.compute_per_token + 2.0e-3
    out, meas = fit_constants(cm, CFG, g, ctx, t_d, t_v, 1.2e-4, 6.0e-4, 2, 1.5)
    assert out.fixed_draft == pytest.approx(1.5e-3, rel=1e-9)
    assert out.fixed_verify == pytest.approx(2.0e-3, rel=1e-9)
    assert out.resync_per_token == pytest.approx(1.2e-4 / 1.5)
    assert out.rebuild_per_token == pytest.approx(6.0e-4 / (ctx * 2 / 32))
    # the device-measured rebuild rate prices a switch, not the resync rate
    assert out.rebuild_cost(ctx) == pytest.approx(ctx * out.rebuild_per_token)
    assert meas["fixed_draft"] == out.fixed_draft
    # a measured time below the byte model clamps at zero
    out, _ = fit_constants(cm, CFG, g, ctx, 1e-6, 1e-6, 0.0, 0.0, 2, 1.0)
    assert out.fixed_draft == 0.0 and out.fixed_verify == 0.0 and out.rebuild_per_token is None


def test_ceiling_reflects_the_measured_overheads():
    """Draft-step overheads lower the ceiling, verify-pass overheads raise it."""
    cm = _cm()
    ctx, c4 = 32768, CompressionConfig(4, 0.25)
    t_v = cm.t_verify(ctx, 1) - cm.fixed_verify
    slow_draft, _ = fit_constants(cm, CFG, 1, ctx, cm.t_draft(CFG, ctx) + 1e-3, t_v, 0.0, 0.0, 2, 1.5)
    slow_verify, _ = fit_constants(cm, CFG, 1, ctx, cm.t_draft(CFG, ctx) - cm.fixed_draft, t_v + 1e-3, 0.0, 0.0,
                                   2, 1.5)
    assert slow_draft.ceiling(c4, ctx) < cm.ceiling(c4, ctx) < slow_verify.ceiling(c4, ctx)


def test_controller_gates_drafting_on_the_calibrated_costs():
    """The same acceptance history drafts under cheap fixed costs and stops
    drafting when the calibrated draft step costs as much as a verify pass."""
    ctx = 32768
    base = _cm()
    cheap, _ = fit_constants(base, CFG, 1, ctx, base.t_draft(CFG, ctx), base.t_verify(ctx, 1), 1e-5, 1e-3, 2, 2.0)
    dear, _ = fit_constants(base, CFG, 1, ctx, base.t_verify(ctx, 1) * 1.2, base.t_verify(ctx, 1), 1e-5, 1e-3, 2,
                            2.0)
    arms = [CFG]
    picks = {}
    for name, cm in (("cheap", cheap), ("dear", dear)):
        ctrl = ThompsonController(cm, arms, gamma_max=8, seed=0)
        gs = []
        for _ in range(60):
            c, g = ctrl.select(ctx, None)
            ctrl.update(c, g, g, ctx, None)        # every draft accepted
            gs.append(g)
        picks[name] = gs[-20:]
    assert min(picks["cheap"]) > 0
    assert max(picks["dear"]) == 0
