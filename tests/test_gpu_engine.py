"""Decode-step parity on the GPU: logits against the oracle, token streams
against the reference's recorded streams and the GPU's own full-KV decode
(losslessness), batching, and the sampling distribution.

Tolerances (max |device - oracle| / max |oracle| over a logits block):
fp32 configs 1e-3, bf16 configs 2e-2.
"""

import json

import numpy as np
import pytest

import oracle
from draftkv.config import CompressionConfig, default_arms
from draftkv.controller import FixedPolicy, ThompsonController
from draftkv.throughput import CostModel
from draftkv import weights as W
from tests.golden.make_golden import ENGINE_CFGS, SMALL_MODELS, small_model_cfg, small_model_weights

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = {"f32": 1e-3, "bf16": 2e-2}


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.loads((golden_dir / "engine_runs.json").read_text()), np.load(golden_dir / "models.npz")


_MODELS = {}


def device_model(name, dtype="f32"):
    key = (name, dtype)
    if key not in _MODELS:
        from draftkv import from_config
        cfg = dict(small_model_cfg(W, name))
        wts = small_model_weights(W, name)
        if dtype == "bf16":
            wts = {k: W.round_bf16(v) for k, v in wts.items()}
        cfg["dtype"] = dtype
        _MODELS[key] = (from_config(wts, cfg), oracle.OracleModel(wts, small_model_cfg(W, name)))
    return _MODELS[key]


@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_fp32_logits_match_reference(golden, name):
    from draftkv import FullKVCache
    meta, npz = golden
    m, _ = device_model(name)
    prompt = meta[name]["prompt"]
    full = FullKVCache(m.n_layers)
    got = m.forward(np.array(prompt[:-1]), full, 0).cpu().numpy()
    assert rel_err(got, npz[f"{name}_prefill"]) < TOL["f32"]
    got = m.forward(np.array([prompt[-1]]), full, len(prompt) - 1).cpu().numpy()
    assert rel_err(got, npz[f"{name}_next"]) < TOL["f32"]
    got = m.forward(np.array([3, 7, 11, 13]), full, len(prompt)).cpu().numpy()
    assert rel_err(got, npz[f"{name}_block"]) < TOL["f32"]


@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_bf16_logits_match_oracle(golden, name):
    from draftkv import FullKVCache
    meta, _ = golden
    m, om = device_model(name, "bf16")
    prompt = meta[name]["prompt"]
    full = FullKVCache(m.n_layers)
    ofull = oracle.OracleFull(m.n_layers)
    got = m.forward(np.array(prompt), full, 0).cpu().numpy()
    want = om.forward(np.array(prompt), ofull, 0)
    assert rel_err(got, want) < TOL["bf16"]


@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_verify_rows_equal_decode_rows(golden, name):
    """A T-token forward gives bit-identical logits to T one-token forwards
    (this is what makes the verify pass reproduce plain decoding)."""
    from draftkv import FullKVCache
    meta, _ = golden
    for dtype in ("f32", "bf16"):
        m, _ = device_model(name, dtype)
        prompt = meta[name]["prompt"]
        a, b = FullKVCache(m.n_layers), FullKVCache(m.n_layers)
        m.forward(np.array(prompt[:-5]), a, 0)
        m.forward(np.array(prompt[:-5]), b, 0)
        blk = m.forward(np.array(prompt[-5:]), a, len(prompt) - 5)
        rows = [m.forward(np.array([t]), b, len(prompt) - 5 + i) for i, t in enumerate(prompt[-5:])]
        for i in range(5):
            assert torch.equal(blk[i], rows[i][0]), (dtype, i)


@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_baseline_tokens_match_reference(golden, name):
    from draftkv import DraftKVEngine
    meta, _ = golden
    m, _ = device_model(name)
    rec = meta[name]
    assert DraftKVEngine(m, seed=0).generate_baseline(rec["prompt"], 24, 0.0) == rec["baseline"]


@pytest.mark.parametrize("name", list(SMALL_MODELS))
@pytest.mark.parametrize("bits,keep", ENGINE_CFGS)
@pytest.mark.parametrize("gamma", [1, 3])
def test_greedy_generate_is_lossless(golden, name, bits, keep, gamma):
    """Reference tests/test_lossless.py:28-35 on the device, with the reference's
    recorded token stream as the target."""
    from draftkv import DraftKVEngine
    meta, _ = golden
    m, _ = device_model(name)
    rec = meta[name]
    r = DraftKVEngine(m, FixedPolicy(CompressionConfig(bits, keep), gamma), seed=0).generate(rec["prompt"], 24, 0.0)
    assert r.tokens == rec["baseline"]
    assert r.new_tokens == 24 and r.verify_passes <= 24


@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_bf16_generate_equals_own_baseline(golden, name):
    from draftkv import DraftKVEngine
    meta, _ = golden
    m, _ = device_model(name, "bf16")
    prompt = meta[name]["prompt"]
    base = DraftKVEngine(m, seed=0).generate_baseline(prompt, 24, 0.0)
    for bits, keep in ((4, 0.5), (2, 0.25), (8, 1.0)):
        r = DraftKVEngine(m, FixedPolicy(CompressionConfig(bits, keep), 4), seed=0).generate(prompt, 24, 0.0)
        assert r.tokens == base, (bits, keep)


@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_controller_driven_run_is_lossless(golden, name):
    """Reference tests/test_lossless.py:49-57: config switches rebuild layers."""
    from draftkv import DraftKVEngine
    meta, _ = golden
    m, _ = device_model(name)
    rec = meta[name]
    cm = CostModel(n_layers=m.n_layers, n_kv_heads=m.n_kv_heads, d_head=m.d_head, weight_bytes=2.0e6,
                   bandwidth=2.0e10, full_kv_bandwidth=6.4e8, hbm_kv_budget=2.0e4)
    r = DraftKVEngine(m, ThompsonController(cm, default_arms(), seed=3), seed=0).generate(rec["prompt"], 24, 0.0)
    assert r.tokens == rec["baseline"]
    assert r.cache_rebuilds >= 2


def test_compression_costs_acceptance(golden):
    """Reference tests/test_lossless.py:38-46: guards against a vacuous suite."""
    from draftkv import DraftKVEngine
    meta, _ = golden
    m, _ = device_model("gpt2_small")
    p = meta["gpt2_small"]["prompt"]
    mild = DraftKVEngine(m, FixedPolicy(CompressionConfig(16, 1.0), 3), seed=0).generate(p, 24, 0.0)
    harsh = DraftKVEngine(m, FixedPolicy(CompressionConfig(2, 0.25), 3), seed=0).generate(p, 24, 0.0)
    assert mild.acceptance_rate > harsh.acceptance_rate + 0.2


def test_batch_matches_single_sequences(golden):
    from draftkv import DraftKVEngine
    meta, _ = golden
    m, _ = device_model("llama_small")
    prompts = [W.tokens(40, m.vocab_size, seed=s) for s in (21, 22, 23)]
    eng = DraftKVEngine(m, FixedPolicy(CompressionConfig(4, 0.5), 3), seed=0)
    res = eng.generate_batch(prompts, 20, 0.0)
    base = DraftKVEngine(m, seed=0).generate_baseline_batch(prompts, 20, 0.0)
    for b in range(3):
        assert res[b].tokens == base[b]
        assert base[b] == DraftKVEngine(m, seed=0).generate_baseline(prompts[b], 20, 0.0)


def test_switch_to_a_wider_arm_regrows_the_drafter_cache(golden):
    """A session whose policy moves to an arm with wider codes and a larger
    budget than its drafter cache was sized for (4-bit keep 0.25, then 8-bit
    keep 1): the cache is re-created and rebuilt, and the tokens still equal
    full-KV decoding."""
    from draftkv import DraftKVEngine
    m, _ = device_model("llama_small")
    prompts = [W.tokens(60, m.vocab_size, seed=s) for s in (31, 32)]
    eng = DraftKVEngine(m, FixedPolicy(CompressionConfig(4, 0.25), 3), seed=0)
    sess = eng.session(prompts, 40, 0.0)
    for _ in range(3):
        sess.round()
    small = sess.st.comp
    eng.controller = FixedPolicy(CompressionConfig(8, 1.0), 3)
    while not sess.done:
        sess.round()
    sess.finish()
    assert sess.st.comp is not small and sess.st.comp.cb_max > small.cb_max and sess.st.comp.cap > small.cap
    base = DraftKVEngine(m, seed=0).generate_baseline_batch(prompts, 40, 0.0)
    for b in range(2):
        assert sess.results()[b].tokens == base[b]


def _tv(a, b):
    return 0.5 * float(np.abs(a - b).sum())


@pytest.mark.parametrize("cfg", [CompressionConfig(8, 1.0), CompressionConfig(2, 0.25)], ids=lambda c: c.label())
def test_first_sampled_token_matches_target_distribution(golden, cfg):
    """Reference tests/test_sampling.py:17-42 (distributional parity): the
    first emitted token's empirical distribution vs exact p, with a control."""
    from draftkv import DraftKVEngine
    meta, _ = golden
    m, om = device_model("llama_small")
    prompt = meta["llama_small"]["prompt"][:24]
    ofull = oracle.OracleFull(om.n_layers)
    om.forward(np.array(prompt[:-1]), ofull, 0)
    p = oracle.probs_of(om.forward(np.array([prompt[-1]]), ofull, len(prompt) - 1)[-1], 1.0)
    # max_new_tokens=5 makes the first round draft 4 tokens, so the first
    # emitted token comes out of acceptance / residual resampling
    trials, batch = 4096, 512
    counts = np.zeros(m.vocab_size)
    for rep in range(trials // batch):
        eng = DraftKVEngine(m, FixedPolicy(cfg, 4), seed=100 + rep)
        for r in eng.generate_batch([prompt] * batch, 5, 1.0):
            counts[r.tokens[len(prompt)]] += 1
    emp = counts / trials
    ctrl = np.bincount(np.random.default_rng(2).choice(m.vocab_size, size=trials, p=p),
                       minlength=m.vocab_size) / trials
    assert _tv(emp, p) < max(1.5 * _tv(ctrl, p), 0.05)


def test_sampling_uses_the_residual_branch(golden):
    """Reference tests/test_sampling.py:45-54."""
    from draftkv import DraftKVEngine
    meta, _ = golden
    m, _ = device_model("gpt2_small")
    r = DraftKVEngine(m, FixedPolicy(CompressionConfig(2, 0.25), 6), seed=4).generate(
        meta["gpt2_small"]["prompt"], 40, 1.0)
    assert r.acceptance_rate < 1.0
    assert r.new_tokens >= 40


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_host_resident_full_cache_is_identical(golden, dtype):
    """Configuration 5's layout: the full cache in pinned host memory (read and
    written by the kernels over the host link), the drafter cache in HBM.
    Same kernels, same arithmetic: token streams and acceptance identical to
    the device-resident run, and equal to full-KV decoding."""
    from draftkv import DraftKVEngine
    meta, _ = golden
    m, _ = device_model("llama_small", dtype)
    prompt = meta["llama_small"]["prompt"]
    pol = lambda: FixedPolicy(CompressionConfig(4, 0.25), 3)  # noqa: E731
    dev = DraftKVEngine(m, pol(), seed=0).generate(prompt, 24, 0.0)
    eng = DraftKVEngine(m, pol(), seed=0)
    eng.offload_full = True
    host = eng.generate(prompt, 24, 0.0)
    assert host.tokens == dev.tokens
    assert [r.accepted for r in host.rounds] == [r.accepted for r in dev.rounds]
    base = DraftKVEngine(m, seed=0)
    base.offload_full = True
    assert base.generate_baseline(prompt, 24, 0.0) == dev.tokens


# ---------------------------------------------------------------- per-layer plans
def _four_layer_llama():
    from draftkv import from_config
    cfg = W.llama_config(4, 128, 4, 2, 192, 101, head_dim=64, tied=True, dtype="f32")
    return from_config(W.make_weights(cfg, seed=5, std=0.09, attn_gain=3.0, attn_sharpness=3.0), cfg)


def test_adaptive_layer_plans_are_lossless_and_rebuild_only_changed_layers():
    """Reference tests/test_adaptive.py:130-171 on the device.  The adaptive
    allocator probes swaps on almost every round (probe_prob 0.9) and
    re-solves its plan every 5 decisions; the greedy stream must equal plain
    full-KV decoding, and every plan change must rebuild exactly the layers
    whose configuration changed."""
    from draftkv import AdaptiveLayerController, DraftKVEngine, LayerPlan
    m = _four_layer_llama()
    prompt = W.tokens(192, m.vocab_size, seed=3)
    base = DraftKVEngine(m, seed=0).generate_baseline(prompt, 32, 0.0)
    cands = [CompressionConfig(4, 0.25), CompressionConfig(4, 0.5), CompressionConfig(4, 1.0)]
    cm = CostModel(n_layers=m.n_layers, n_kv_heads=m.n_kv_heads, d_head=m.d_head, weight_bytes=2.0e6,
                   bandwidth=2.0e10, full_kv_bandwidth=6.4e8, hbm_kv_budget=2.0e5)
    lo = LayerPlan.uniform(cands[0], m.n_layers).per_layer_bytes(256, m.n_kv_heads, m.d_head)
    hi = LayerPlan.uniform(cands[-1], m.n_layers).per_layer_bytes(256, m.n_kv_heads, m.d_head)
    ctrl = AdaptiveLayerController(cm, m.n_layers, lo + 0.5 * (hi - lo), cands, ctx_hint=256, probe_prob=0.9,
                                   resolve_every=5, seed=3)
    eng = DraftKVEngine(m, ctrl, seed=0)
    calls, plans = [], []
    real = eng._rebuild

    def spy(st, layers, ctx_t, advance):
        calls.append(list(layers))
        plans.append(list(st.comp.cfgs))
        real(st, layers, ctx_t, advance)

    eng._rebuild = spy
    r = eng.generate(prompt, 32, 0.0)
    assert r.tokens == base
    assert ctrl.n_probes > 0 and r.cache_rebuilds >= 3
    assert calls[0] == list(range(m.n_layers))          # first sync: every layer
    for prev, cur, layers in zip(plans, plans[1:], calls[1:]):
        assert layers and layers == [L for L in range(m.n_layers) if prev[L] != cur[L]]


def test_partial_rebuild_leaves_other_layers_untouched():
    """Reference tests/test_adaptive.py:130-150: rebuilding one layer for a
    new configuration rewrites that layer only (device cache, read back)."""
    from draftkv import CompressedKVCache, FullKVCache
    m = _four_layer_llama()
    toks = np.arange(64) % m.vocab_size
    full = FullKVCache(m.n_layers)
    m.forward(toks, full, 0)
    comp = CompressedKVCache(m.n_layers, CompressionConfig(4, 1.0))
    comp.materialize(m.n_kv_heads, m.d_head, m.dtype)
    comp.sync_from(full, 0)
    before = [comp.read(L)[0].copy() for L in range(m.n_layers)]
    cfgs = [CompressionConfig(4, 1.0)] * m.n_layers
    cfgs[1] = CompressionConfig(4, 0.25)
    rows = comp.rebuild_layers(full, [1], cfgs)
    assert rows == 64
    assert comp.cfgs[1] == CompressionConfig(4, 0.25)
    for L in range(m.n_layers):
        assert np.array_equal(comp.read(L)[0], before[L]) == (L != 1), L


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("name", list(SMALL_MODELS))
def test_checkpoint_directory_matches_oracle(tmp_path, golden, name, dtype):
    """A HuggingFace-style directory (config.json + model.safetensors, fp32 or
    bf16 tensors) through from_dir, against the oracle fed the reference
    reader's decoding of the same file (fp32 numpy): logits within the
    configuration's tolerance."""
    from draftkv import FullKVCache, GPT2, LlamaLike
    from draftkv.checkpoint import load_safetensors, save_safetensors
    meta, _ = golden
    cfg = {k: v for k, v in small_model_cfg(W, name).items() if k != "dtype"}
    cfg["torch_dtype"] = "bfloat16" if dtype == "bf16" else "float32"
    wts = small_model_weights(W, name)
    if dtype == "bf16":
        wts = {k: torch.from_numpy(v).to(torch.bfloat16) for k, v in wts.items()}
    save_safetensors(wts, tmp_path / "model.safetensors", metadata={"format": "pt"})
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    m = (GPT2 if "n_embd" in cfg else LlamaLike).from_dir(tmp_path)
    assert (m.dtype == 1) == (dtype == "bf16")
    om = oracle.OracleModel(load_safetensors(tmp_path / "model.safetensors"), cfg)
    prompt = meta[name]["prompt"]
    got = m.forward(np.array(prompt), FullKVCache(m.n_layers), 0).cpu().numpy()
    want = om.forward(np.array(prompt), oracle.OracleFull(om.n_layers), 0)
    assert rel_err(got, want) < TOL[dtype]
