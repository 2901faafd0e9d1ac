"""Host policy parity: config byte accounting, cost model and controller
decisions against values recorded from the reference (tests/golden/policy.json),
plus the reference's own math properties (reference tests/test_math.py)."""

import json

import numpy as np
import pytest

from draftkv.config import CompressionConfig, LayerPlan, default_arms
from draftkv.controller import DepthThompsonController, ThompsonController
from draftkv.throughput import (CostModel, best_gamma, expected_tokens,
                                expected_tokens_profile)


@pytest.fixture(scope="module")
def policy(golden_dir):
    return json.loads((golden_dir / "policy.json").read_text())


def test_cost_model_grid(policy):
    cm = CostModel(n_layers=32, n_kv_heads=8, d_head=128, weight_bytes=15.0e9,
                   bandwidth=6.5e12, batch=4)
    for r in policy["grid"]:
        c = CompressionConfig(r["bits"], r["keep"])
        ctx = r["ctx"]
        assert cm.ceiling(c, ctx) == r["ceiling"]
        assert cm.t_draft(c, ctx) == r["t_draft"]
        assert cm.t_verify(ctx, 4) == r["t_verify"]
        assert cm.t_baseline(ctx) == r["t_base"]
        assert cm.rebuild_cost(ctx) == r["rebuild"]
        assert list(best_gamma(cm, c, 0.8, ctx, 8)) == r["best"]
        assert c.bytes_per_entry(128) == r["bpe"]


@pytest.mark.parametrize("kind", ["thompson", "depth"])
def test_controller_traces(policy, kind):
    cm = CostModel(full_kv_bandwidth=6.4e10, hbm_kv_budget=1e9)
    ctrl = (ThompsonController(cm, default_arms(), seed=5) if kind == "thompson"
            else DepthThompsonController(cm, default_arms(), seed=5))
    rng = np.random.default_rng(12)
    for rd, want in enumerate(policy["traces"][kind]):
        ctx = 32768 + 17 * rd
        c, g = ctrl.select(ctx, None)
        k = 0
        a = 0.95 if c.bits >= 8 else (0.8 if c.bits == 4 else 0.4)
        while k < g and rng.random() < a:
            k += 1
        ctrl.update(c, g, k, ctx, None)
        assert [c.bits, c.keep_frac, g, k] == want, rd


def test_misc(policy):
    m = policy["misc"]
    for a, g, e in m["E"]:
        assert expected_tokens(a, g) == e
    for prof, e in m["Eprof"]:
        assert expected_tokens_profile(prof) == e
    assert [[c.bits, c.keep_frac] for c in default_arms()] == m["arms"]
    plan = LayerPlan((CompressionConfig(4, 0.5), CompressionConfig(2, 0.25), CompressionConfig(16, 1.0)))
    assert plan.per_layer_bytes(1000, 8, 128) == m["plan_bytes"]


def test_config_validation():
    with pytest.raises(ValueError):
        CompressionConfig(5, 0.5)
    with pytest.raises(ValueError):
        CompressionConfig(4, 0.0)
    assert CompressionConfig(16, 1.0).lossless and not CompressionConfig(8, 1.0).lossless


# ---- reference tests/test_math.py properties
def test_speedup_never_exceeds_ceiling():
    cm = CostModel(full_kv_bandwidth=6.4e10, hbm_kv_budget=1e9)
    for ctx in (512, 8192, 131072):
        for cfg in (CompressionConfig(16, 1.0), CompressionConfig(4, 0.5), CompressionConfig(2, 0.25)):
            ceil = cm.ceiling(cfg, ctx)
            for g in range(1, 32):
                assert cm.speedup(cfg, g, 0.999, ctx) <= ceil + 1e-9


def test_best_gamma_monotone_in_alpha():
    cm = CostModel(full_kv_bandwidth=6.4e10, hbm_kv_budget=1e9)
    gs = [best_gamma(cm, CompressionConfig(4, 0.5), a, 32768, 16)[0]
          for a in (0.1, 0.3, 0.5, 0.7, 0.9, 0.99)]
    assert gs == sorted(gs)


def test_expected_tokens_saturates():
    for a in (0.5, 0.8, 0.95):
        assert expected_tokens(a, 1000) == pytest.approx(1 / (1 - a), rel=1e-6)
