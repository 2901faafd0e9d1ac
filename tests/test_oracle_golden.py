"""Pin the CPU oracle to golden vectors produced by the reference itself.

tests/golden/make_golden.py imported the reference package and recorded its
outputs; here the oracle (oracle/) must reproduce them: quantize bit-exact,
eviction states exactly, logits to fp32 round-off, token streams and
acceptance traces exactly (including temperature-1 sampling, whose random
draws the oracle consumes in the reference's order).
"""

import json

import numpy as np
import pytest

import oracle
from oracle.caches import OracleComp, OraclePaged
from draftkv.config import CompressionConfig, default_arms
from draftkv.controller import FixedPolicy, ThompsonController
from draftkv.throughput import CostModel
from tests.golden.make_golden import (ENGINE_CFGS, QUANT_CASES, SMALL_MODELS,
                                      small_model_cfg, small_model_weights)
from draftkv import weights as W


@pytest.fixture(scope="module")
def quant_npz(golden_dir):
    return np.load(golden_dir / "quantize.npz")


@pytest.mark.parametrize("cid", [c for _, c in QUANT_CASES])
@pytest.mark.parametrize("bits", [2, 3, 4, 8, 16])
def test_quantize_bit_exact(quant_npz, cid, bits):
    x = quant_npz[f"x{cid}"]
    want = quant_npz[f"deq{cid}_b{bits}"]
    got = oracle.quantize(x, bits)
    assert got.dtype == want.dtype and got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_codes_reconstruct_the_dequantized_values(quant_npz):
    x = quant_npz["x1"]
    for bits in (2, 3, 4, 8):
        codes, scale, lo, deq = oracle.quant_codes(x, bits)
        assert codes.max() <= (1 << bits) - 1
        g = codes.reshape(codes.shape[0], -1, 64).astype(np.float32)
        rec = (g * scale[..., None] + lo[..., None]).reshape(codes.shape[0], -1)
        assert np.array_equal(rec[:, : x.shape[-1]].reshape(x.shape), deq)


def test_eviction_trace(golden_dir):
    states = json.loads((golden_dir / "evict_trace.json").read_text())["states"]
    comp = OracleComp(2, CompressionConfig(bits=4, keep_frac=0.5, sink=2, recent=4))
    rng = np.random.default_rng(7)
    pos = 0
    for step, want in enumerate(states):
        n_rows = 1 if step % 7 else 3
        for L in range(2):
            k = rng.standard_normal((n_rows, 2, 64)).astype(np.float32)
            v = rng.standard_normal((n_rows, 2, 64)).astype(np.float32)
            comp.append(L, k, v, np.arange(pos, pos + n_rows))
            probs = rng.random((1, 2, len(comp.pos[L]))).astype(np.float32)
            probs /= probs.sum(-1, keepdims=True)
            comp.note_attention(L, probs)
        pos += n_rows
        if step % 9 == 8:
            pos -= 2
            comp.truncate(pos)
        assert comp.pos == want["pos"], step
        assert comp.seen == want["seen"]
        for L in range(2):
            assert comp.score[L] == pytest.approx(want["score"][L], rel=0, abs=0)


@pytest.fixture(scope="module")
def engine_golden(golden_dir):
    return (json.loads((golden_dir / "engine_runs.json").read_text()),
            np.load(golden_dir / "models.npz"))


def _oracle_model(name):
    return oracle.OracleModel(small_model_weights(W, name), small_model_cfg(W, name))


@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_logits(engine_golden, name):
    meta, npz = engine_golden
    m = _oracle_model(name)
    prompt = meta[name]["prompt"]
    full = oracle.OracleFull(m.n_layers)
    np.testing.assert_allclose(m.forward(np.array(prompt[:-1]), full, 0),
                               npz[f"{name}_prefill"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(m.forward(np.array([prompt[-1]]), full, len(prompt) - 1),
                               npz[f"{name}_next"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(m.forward(np.array([3, 7, 11, 13]), full, len(prompt)),
                               npz[f"{name}_block"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_engine_token_streams(engine_golden, name):
    meta, _ = engine_golden
    m = _oracle_model(name)
    rec = meta[name]
    prompt = rec["prompt"]
    assert oracle.OracleEngine(m, None, seed=0).generate_baseline(prompt, 24, 0.0) == rec["baseline"]
    assert oracle.OracleEngine(m, None, seed=9).generate_baseline(prompt, 12, 1.0) == rec["sample_baseline"]
    for bits, keep in ENGINE_CFGS:
        for g in (1, 3):
            want = rec["runs"][f"b{bits}_k{keep}_g{g}"]
            r = oracle.OracleEngine(m, FixedPolicy(CompressionConfig(bits, keep), g), seed=0).generate(prompt, 24, 0.0)
            assert r.tokens == want["tokens"] == rec["baseline"]
            assert [x.accepted for x in r.rounds] == want["k"], (bits, keep, g)
    want = rec["runs"]["sample_b4_k0.5_g3"]
    r = oracle.OracleEngine(m, FixedPolicy(CompressionConfig(4, 0.5), 3), seed=4).generate(prompt, 16, 1.0)
    assert r.tokens == want["tokens"] and [x.accepted for x in r.rounds] == want["k"]


@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_engine_with_controller_and_paged_cache(engine_golden, name):
    meta, _ = engine_golden
    m = _oracle_model(name)
    rec = meta[name]
    prompt = rec["prompt"]
    cm = CostModel(n_layers=m.n_layers, n_kv_heads=m.n_kv_heads, d_head=m.d_head,
                   weight_bytes=2.0e6, bandwidth=2.0e10, full_kv_bandwidth=6.4e8,
                   hbm_kv_budget=2.0e4)
    r = oracle.OracleEngine(m, ThompsonController(cm, default_arms(), seed=3), seed=0).generate(prompt, 24, 0.0)
    want = rec["runs"]["thompson"]
    assert r.tokens == want["tokens"]
    assert [x.accepted for x in r.rounds] == want["k"]
    assert [[x.cfg.bits, x.cfg.keep_frac] for x in r.rounds] == want["cfgs"]
    assert r.cache_rebuilds == want["rebuilds"]
    eng = oracle.OracleEngine(m, FixedPolicy(CompressionConfig(4, 0.5), 3), seed=0,
                              full_factory=lambda: OraclePaged(m.n_layers, m.n_kv_heads, m.d_head, 4, 4096))
    r = eng.generate(prompt, 24, 0.0)
    want = rec["runs"]["paged_b4_k0.5_g3"]
    assert r.tokens == want["tokens"] and [x.accepted for x in r.rounds] == want["k"]


def test_paged_trace(golden_dir):
    trace = json.loads((golden_dir / "paged_trace.json").read_text())
    pk = OraclePaged(2, 2, 64, block_size=4, n_blocks=64)
    n = 0
    for st in trace:
        t = st["t"]
        for L in range(2):
            pk.append(L, np.zeros((t, 2, 64)), np.zeros((t, 2, 64)), np.arange(n, n + t))
        n += t
        if st["cut"] is not None:
            n = st["cut"]
            pk.truncate(n)
        assert n == st["n"]
        assert pk.table == st["tables"]
        assert pk.pool.free_list == st["free"]
