"""The device-calibrated cost model (draftkv/calibrate.py): the constants fitted
from measured phase times, and controllers consuming them (CPU only: the
timings are given, the GPU run measures them in bench.py)."""

import pytest

from draftkv import CompressionConfig, CostModel, ThompsonController
from draftkv.calibrate import fit_constants

CFG = CompressionConfig(8, 1.0)
CTX = 32768


def _cm(**kw):
    return CostModel(n_layers=32, n_kv_heads=8, d_head=128, weight_bytes=15.0e9, bandwidth=6.5e12, batch=4, **kw)


def _times(cm, bw, extra_draft, gamma=2):
    t_d = (cm.weight_bytes + cm.draft_kv_bytes(CFG, CTX)) / bw + extra_draft
    t_v = (cm.weight_bytes + cm.full_kv_bytes(CTX)) / bw
    return t_d, t_v


def test_fit_recovers_the_effective_rate_and_the_draft_overhead():
    cm = _cm()
    t_d, t_v = _times(cm, 4.3e12, 1.5e-3)
    out, meas = fit_constants(cm, CFG, 2, CTX, t_d, t_v, 1.2e-4, 6.0e-4, 2, 1.5)
    assert out.bandwidth == pytest.approx(4.3e12) and out.full_kv_bandwidth == pytest.approx(4.3e12)
    assert out.fixed_draft == pytest.approx(1.5e-3, rel=1e-9) and out.fixed_verify == 0.0
    assert out.compute_per_token == 0.0
    assert out.t_verify(CTX, 2) == pytest.approx(t_v) and out.t_draft(CFG, CTX) == pytest.approx(t_d)
    assert out.resync_per_token == pytest.approx(1.2e-4 / 1.5)
    assert out.rebuild_per_token == pytest.approx(6.0e-4 / (CTX * 2 / 32))
    # the device-measured rebuild rate prices a switch, not the resync rate
    assert out.rebuild_cost(CTX) == pytest.approx(CTX * out.rebuild_per_token)
    assert meas["bandwidth"] == out.bandwidth
    # a draft step faster than the verify pass's rate: no negative offset
    out, _ = fit_constants(cm, CFG, 2, CTX, t_d * 0.5, t_v, 0.0, 0.0, 2, 1.0)
    assert out.fixed_draft == 0.0 and out.rebuild_per_token is None


def test_a_16bit_drafter_kept_whole_cannot_pay():
    """Calibrated on the 8-bit arm, the model prices the 16-bit keep-1 arm at
    the verify pass's own rate: its ceiling is 1 (it never pays), while the
    evicting 4-bit arm keeps a ceiling well above 1."""
    cm = _cm()
    out, _ = fit_constants(cm, CFG, 2, CTX, *_times(cm, 4.3e12, 0.0), 0.0, 0.0, 2, 1.5)
    assert out.ceiling(CompressionConfig(16, 1.0), CTX) == pytest.approx(1.0, abs=1e-9)
    assert out.ceiling(CompressionConfig(4, 0.25), CTX) > 1.8


def test_offloaded_full_cache_keeps_the_link_rate():
    cm = _cm(full_kv_bandwidth=5.0e10)
    t_d = (cm.weight_bytes + cm.draft_kv_bytes(CFG, CTX)) / 4.0e12
    t_v = cm.weight_bytes / 4.0e12 + cm.full_kv_bytes(CTX) / 5.0e10 + 2e-3
    out, _ = fit_constants(cm, CFG, 2, CTX, t_d, t_v, 0.0, 0.0, 2, 1.0)
    assert out.bandwidth == pytest.approx(4.0e12) and out.full_kv_bandwidth == 5.0e10
    assert out.fixed_verify == pytest.approx(2e-3) and out.fixed_draft == 0.0


def test_controller_gates_drafting_on_the_calibrated_costs():
    """The same acceptance history drafts when the measured draft step is
    cheap and stops drafting when it costs as much as a verify pass."""
    base = _cm()
    cheap, _ = fit_constants(base, CFG, 1, CTX, *_times(base, 4.3e12, 0.0), 1e-5, 1e-3, 2, 2.0)
    t_d, t_v = _times(base, 4.3e12, 0.0)
    dear, _ = fit_constants(base, CFG, 1, CTX, t_v * 1.2, t_v, 1e-5, 1e-3, 2, 2.0)
    picks = {}
    for name, cm in (("cheap", cheap), ("dear", dear)):
        ctrl = ThompsonController(cm, [CFG], gamma_max=8, seed=0)
        gs = []
        for _ in range(60):
            c, g = ctrl.select(CTX, None)
            ctrl.update(c, g, g, CTX, None)        # every draft accepted
            gs.append(g)
        picks[name] = gs[-20:]
    assert min(picks["cheap"]) > 0
    assert max(picks["dear"]) == 0
