"""Generate golden fixtures by running the reference implementation itself.

Run in a container that has the reference checkout (pure python + numpy):

    python tests/golden/make_golden.py --reference <path to Draft-KV checkout>

It imports the reference's `draftkv` package, feeds it the seeded inputs
defined here (weights from draft-kv_b200/draftkv/weights.py, loaded by file
path so the two packages named `draftkv` never meet), and writes the inputs'
seeds and the reference outputs to tests/golden/*.npz / *.json.  The tests pin
the CPU oracle (oracle/) to these files; the GPU tests then compare the device
path to the oracle.  Nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent

# ---------------------------------------------------------------- cases
# Small model shapes used across the fixtures (and by the GPU parity tests).
SMALL_MODELS = {
    "gpt2_small": dict(kind="gpt2", n_layers=2, d_model=128, n_heads=2, vocab=97,
                       n_positions=256, seed=3, std=0.09, gain=3.0, sharp=3.0),
    "llama_small": dict(kind="llama", n_layers=2, d_model=128, n_heads=4, n_kv=2,
                        head_dim=64, d_ff=192, vocab=101, theta=10000.0, seed=5,
                        std=0.09, gain=3.0, sharp=3.0),
}

QUANT_CASES = [((7, 3, 64), 0), ((5, 2, 128), 1), ((4, 1, 100), 2), ((3, 2, 8), 3),
               ((6, 2, 64), 4)]
ENGINE_CFGS = [(16, 1.0), (8, 1.0), (4, 1.0), (4, 0.5), (3, 0.5), (2, 0.25)]


def load_weights_module():
    spec = importlib.util.spec_from_file_location(
        "dkv_weights", REPO / "draft-kv_b200" / "draftkv" / "weights.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def small_model_cfg(W, name):
    s = SMALL_MODELS[name]
    if s["kind"] == "gpt2":
        cfg = W.gpt2_config(s["n_layers"], s["d_model"], s["n_heads"], s["vocab"],
                            n_positions=s["n_positions"])
    else:
        cfg = W.llama_config(s["n_layers"], s["d_model"], s["n_heads"], s["n_kv"],
                             s["d_ff"], s["vocab"], head_dim=s["head_dim"],
                             theta=s["theta"], tied=True, dtype="f32")
    return cfg


def small_model_weights(W, name):
    s = SMALL_MODELS[name]
    return W.make_weights(small_model_cfg(W, name), seed=s["seed"], std=s["std"],
                          attn_gain=s["gain"], attn_sharpness=s["sharp"])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", choices=["adaptive", "safetensors"], default=None,
                    help="write only this fixture (the others are left as they are)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    import draftkv as ref                          # the reference package
    if args.only == "adaptive":
        adaptive_fixtures(ref)
        return
    if args.only == "safetensors":
        safetensors_fixture()
        return
    from draftkv import compress as rc
    from draftkv.gpt2 import GPT2
    from draftkv.llama import LlamaLike
    from draftkv.paged import PagedKVCache
    W = load_weights_module()
    out = {}

    # ---- 1. quantize (compress.py:21-46): dequantized outputs, bit-exact
    q = {}
    rng = np.random.default_rng(100)
    for shape, cid in QUANT_CASES:
        x = rng.standard_normal(shape).astype(np.float32)
        x[0, 0, :] = 0.75                               # constant row: hi == lo
        if shape[-1] >= 64:
            x[-1, -1, 5] = 40.0                          # outlier channel
        q[f"x{cid}"] = x
        for b in (2, 3, 4, 8, 16):
            q[f"deq{cid}_b{b}"] = rc.quantize(x, b)
    np.savez_compressed(HERE / "quantize.npz", **q)

    # ---- 2. drafter-cache eviction trace (compress.py:122-230)
    trace = []
    cfg = ref.CompressionConfig(bits=4, keep_frac=0.5, sink=2, recent=4)
    comp = rc.CompressedKVCache(2, cfg)
    rng = np.random.default_rng(7)
    pos = 0
    for step in range(40):
        n_rows = 1 if step % 7 else 3
        for L in range(2):
            k = rng.standard_normal((n_rows, 2, 64)).astype(np.float32)
            v = rng.standard_normal((n_rows, 2, 64)).astype(np.float32)
            p = np.arange(pos, pos + n_rows)
            comp.append(L, k, v, p)
            probs = rng.random((1, 2, len(comp.pos[L]))).astype(np.float32)
            probs /= probs.sum(-1, keepdims=True)
            comp.note_attention(L, probs)
        pos += n_rows
        if step % 9 == 8:
            cut = pos - 2
            comp.truncate(cut)
            pos = cut
        trace.append(dict(pos=[list(map(int, comp.pos[L])) for L in range(2)],
                          score=[list(map(float, comp.score[L])) for L in range(2)],
                          seen=int(comp.seen_positions)))
    (HERE / "evict_trace.json").write_text(json.dumps(dict(states=trace)))

    # ---- 3. small models: prefill + decode logits, and engine runs
    eng = {}
    for name in SMALL_MODELS:
        wts = small_model_weights(W, name)
        cfgd = small_model_cfg(W, name)
        model = GPT2(wts, cfgd) if SMALL_MODELS[name]["kind"] == "gpt2" else LlamaLike(wts, cfgd)
        prompt = W.tokens(40, cfgd["vocab_size"], seed=11)
        full = rc.FullKVCache(model.n_layers)
        lg_prefill = model.forward(np.array(prompt[:-1]), full, 0)
        lg_next = model.forward(np.array([prompt[-1]]), full, len(prompt) - 1)
        blk = np.array([3, 7, 11, 13])
        lg_block = model.forward(blk, full, len(prompt))
        rec = dict(prompt=prompt, prefill=lg_prefill, next=lg_next, block=lg_block)
        base = ref.DraftKVEngine(model, seed=0).generate_baseline(prompt, 24, 0.0)
        rec["baseline"] = base
        runs = {}
        for bits, keep in ENGINE_CFGS:
            for gamma in (1, 3):
                pol = ref.FixedPolicy(ref.CompressionConfig(bits, keep), gamma)
                r = ref.DraftKVEngine(model, pol, seed=0).generate(prompt, 24, 0.0)
                runs[f"b{bits}_k{keep}_g{gamma}"] = dict(
                    tokens=r.tokens, k=[x.accepted for x in r.rounds],
                    g=[x.gamma for x in r.rounds], rebuilds=r.cache_rebuilds)
        # sampling (temperature 1): RNG-exact in the oracle
        pol = ref.FixedPolicy(ref.CompressionConfig(4, 0.5), 3)
        r = ref.DraftKVEngine(model, pol, seed=4).generate(prompt, 16, 1.0)
        runs["sample_b4_k0.5_g3"] = dict(tokens=r.tokens, k=[x.accepted for x in r.rounds],
                                         g=[x.gamma for x in r.rounds], rebuilds=r.cache_rebuilds)
        rec["sample_baseline"] = ref.DraftKVEngine(model, seed=9).generate_baseline(prompt, 12, 1.0)
        # controller-driven run (config switches exercise rebuild_layers)
        cm = ref.CostModel(n_layers=model.n_layers, n_kv_heads=model.n_kv_heads if hasattr(model, "n_kv_heads") else model.n_heads,
                           d_head=model.d_head, weight_bytes=2.0e6, bandwidth=2.0e10,
                           full_kv_bandwidth=6.4e8, hbm_kv_budget=2.0e4)
        ctrl = ref.ThompsonController(cm, ref.default_arms(), seed=3)
        r = ref.DraftKVEngine(model, ctrl, seed=0).generate(prompt, 24, 0.0)
        runs["thompson"] = dict(tokens=r.tokens, k=[x.accepted for x in r.rounds],
                                g=[x.gamma for x in r.rounds], rebuilds=r.cache_rebuilds,
                                cfgs=[[x.cfg.bits, x.cfg.keep_frac] for x in r.rounds])
        # paged authoritative cache (paged.py) under the same engine
        pe = ref.DraftKVEngine(model, ref.FixedPolicy(ref.CompressionConfig(4, 0.5), 3), seed=0,
                               full_cache_factory=lambda m=model: PagedKVCache(
                                   m.n_layers, getattr(m, "n_kv_heads", m.n_heads), m.d_head, 4, 4096))
        r = pe.generate(prompt, 24, 0.0)
        runs["paged_b4_k0.5_g3"] = dict(tokens=r.tokens, k=[x.accepted for x in r.rounds],
                                        g=[x.gamma for x in r.rounds], rebuilds=r.cache_rebuilds)
        rec["runs"] = runs
        eng[name] = rec
    npz = {}
    meta = {}
    for name, rec in eng.items():
        for key in ("prefill", "next", "block"):
            npz[f"{name}_{key}"] = rec[key]
        meta[name] = dict(prompt=rec["prompt"], baseline=rec["baseline"],
                          sample_baseline=rec["sample_baseline"], runs=rec["runs"])
    np.savez_compressed(HERE / "models.npz", **npz)
    (HERE / "engine_runs.json").write_text(json.dumps(meta))

    # ---- 4. host policy: controllers and cost model
    cm = ref.CostModel(n_layers=32, n_kv_heads=8, d_head=128, weight_bytes=15.0e9,
                       bandwidth=6.5e12, batch=4)
    grid = []
    for bits, keep in ((16, 1.0), (8, 1.0), (4, 0.5), (4, 0.25), (2, 0.25), (3, 0.5)):
        c = ref.CompressionConfig(bits, keep)
        for ctx in (512, 8192, 32768, 262144):
            grid.append(dict(bits=bits, keep=keep, ctx=ctx, ceiling=cm.ceiling(c, ctx),
                             t_draft=cm.t_draft(c, ctx), t_verify=cm.t_verify(ctx, 4),
                             t_base=cm.t_baseline(ctx), rebuild=cm.rebuild_cost(ctx),
                             best=list(ref.best_gamma(cm, c, 0.8, ctx, 8)),
                             bpe=c.bytes_per_entry(128)))
    cm2 = ref.CostModel(full_kv_bandwidth=6.4e10, hbm_kv_budget=1e9)
    ctrl_traces = {}
    for cname in ("thompson", "depth"):
        if cname == "thompson":
            ctrl = ref.ThompsonController(cm2, ref.default_arms(), seed=5)
        else:
            ctrl = ref.DepthThompsonController(cm2, ref.default_arms(), seed=5)
        rng = np.random.default_rng(12)
        tr = []
        for rd in range(150):
            ctx = 32768 + 17 * rd
            c, g = ctrl.select(ctx, None)
            k = 0
            a = 0.95 if c.bits >= 8 else (0.8 if c.bits == 4 else 0.4)
            while k < g and rng.random() < a:
                k += 1
            ctrl.update(c, g, k, ctx, None)
            tr.append([c.bits, c.keep_frac, g, k])
        ctrl_traces[cname] = tr
    from draftkv.throughput import expected_tokens, expected_tokens_profile
    misc = dict(
        E=[[a, g, expected_tokens(a, g)] for a in (0.0, 0.3, 0.9, 1.0) for g in (0, 1, 5)],
        Eprof=[[[0.5, 0.8, 0.9], expected_tokens_profile([0.5, 0.8, 0.9])]],
        arms=[[c.bits, c.keep_frac] for c in ref.default_arms()],
        plan_bytes=ref.LayerPlan((ref.CompressionConfig(4, 0.5), ref.CompressionConfig(2, 0.25),
                                  ref.CompressionConfig(16, 1.0))).per_layer_bytes(1000, 8, 128),
    )
    (HERE / "policy.json").write_text(json.dumps(dict(grid=grid, traces=ctrl_traces, misc=misc)))

    # ---- 5. paged allocator trace (paged.py:33-177)
    pk = PagedKVCache(2, 2, 64, block_size=4, n_blocks=64)
    rng = np.random.default_rng(21)
    ptrace = []
    n = 0
    for step in range(30):
        t = int(rng.integers(1, 7))
        cut = None
        for L in range(2):
            pk.append(L, rng.standard_normal((t, 2, 64)), rng.standard_normal((t, 2, 64)),
                      np.arange(n, n + t))
        n += t
        if step % 3 == 2:
            n = max(0, n - int(rng.integers(0, 6)))
            pk.truncate(n)
            cut = n
        ptrace.append(dict(t=t, cut=cut, n=n, tables=[list(map(int, pk.block_table[L])) for L in range(2)],
                           free=list(map(int, pk.pool._free)), frag=pk.fragmentation()))
    (HERE / "paged_trace.json").write_text(json.dumps(ptrace))
    adaptive_fixtures(ref)
    safetensors_fixture()
    print("golden fixtures written to", HERE)


def safetensors_fixture():
    """A small safetensors file (F32, F16, BF16, I64 tensors and metadata)
    written by the device build's writer, and what the reference's reader
    (gpt2.py:25-46) decodes from it."""
    import torch
    from draftkv.gpt2 import load_safetensors as ref_load
    spec = importlib.util.spec_from_file_location("dkv_checkpoint", REPO / "draft-kv_b200" / "draftkv" / "checkpoint.py")
    ck = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ck)
    rng = np.random.default_rng(41)
    tensors = {
        "a.f32": rng.standard_normal((3, 5)).astype(np.float32),
        "b.f16": rng.standard_normal((7,)).astype(np.float16),
        "c.bf16": torch.from_numpy(rng.standard_normal((4, 6)).astype(np.float32)).to(torch.bfloat16),
        "d.i64": np.arange(-3, 5, dtype=np.int64).reshape(2, 4),
    }
    path = HERE / "tiny.safetensors"
    ck.save_safetensors(tensors, path, metadata={"format": "pt"})
    got = ref_load(path)
    np.savez_compressed(HERE / "tiny_safetensors_ref.npz", **{k.replace(".", "_"): v for k, v in got.items()})


# ---------------------------------------------------------------- adaptive allocator
ADAPTIVE_NL = 6
ADAPTIVE_CTX = 32768


def adaptive_setup(ref_or_ours, resync=1.0e-7):
    """Candidates, cost model and budget function of the adaptive-allocator
    scenarios (the shapes of the reference's tests/test_adaptive.py:15-35),
    built from either package's CompressionConfig / CostModel / LayerPlan."""
    m = ref_or_ours
    cands = [m.CompressionConfig(4, 0.25), m.CompressionConfig(4, 0.5), m.CompressionConfig(4, 1.0)]
    cm = m.CostModel(n_layers=ADAPTIVE_NL, n_kv_heads=12, d_head=64, weight_bytes=2.0e9,
                     full_kv_bandwidth=6.4e10, hbm_kv_budget=4.0e8, resync_per_token=resync)
    lo = m.LayerPlan.uniform(cands[0], ADAPTIVE_NL).per_layer_bytes(ADAPTIVE_CTX, 12, 64)
    hi = m.LayerPlan.uniform(cands[-1], ADAPTIVE_NL).per_layer_bytes(ADAPTIVE_CTX, 12, 64)
    return cands, cm, (lambda frac: lo + frac * (hi - lo))


# (name, controller kwargs, phases of (env damage, env seed, rounds, key)); a
# phase with env seed None keeps the previous environment and shifts its damage
ADAPTIVE_SCENARIOS = [
    ("find", dict(budget=0.5, probe_prob=0.4, resolve_every=40, seed=2), [({2: 2.5}, 1, 900, None)]),
    ("shift", dict(budget=0.5, probe_prob=0.4, resolve_every=40, decay=0.97, seed=6),
     [({1: 2.5}, 5, 800, None), ({4: 2.5}, None, 1200, None)]),
    ("keys", dict(budget=0.5, probe_prob=0.4, resolve_every=40, seed=7),
     [({0: 2.5}, 8, 700, "prose"), ({5: 2.5}, 9, 700, "code")]),
    ("rate", dict(budget=0.6, probe_prob=0.1, resolve_every=50, seed=11), [({3: 1.0}, 10, 1000, None)]),
    ("stall", dict(budget=0.2, probe_prob=0.3, resolve_every=25, seed=13),
     [({L: 4.0 for L in range(ADAPTIVE_NL)}, 14, 300, None)]),
]


def adaptive_fixtures(ref):
    """Decision logs of the reference's AdaptiveLayerController
    (adaptive.py:68-335) driven by its simulated per-layer environment
    (sim.py:131-167): per round the plan (candidate index per layer), gamma
    and the accepted count the environment returned; plus the reference's
    exact knapsack (layers.py:301-368) on random damage tables and its probe
    throttle."""
    from draftkv.adaptive import AdaptiveLayerController
    from draftkv.layers import SensitivityProfile, allocate
    from draftkv.sim import LayerEnv
    logs = {}
    for name, kw, phases in ADAPTIVE_SCENARIOS:
        cands, cm, budget = adaptive_setup(ref)
        kw = dict(kw)
        ctrl = AdaptiveLayerController(cm, ADAPTIVE_NL, budget(kw.pop("budget")), cands, ctx_hint=ADAPTIVE_CTX, **kw)
        env, rounds = None, []
        for dmg, seed, n, key in phases:
            if seed is None:
                env.shift(dmg)
            else:
                env = LayerEnv(damage=dmg, ranked=cands, ctx=ADAPTIVE_CTX, seed=seed)
            for _ in range(n):
                plan, g = ctrl.select(env.ctx, key)
                k = env.pull(plan, g) if g > 0 else 0
                ctrl.update(plan, g, k, env.ctx, key)
                rounds.append([[cands.index(c) for c in plan], g, k])
        logs[name] = dict(rounds=rounds, damages={str(k): ctrl.damages(k) for k in ctrl.stats},
                          probes=ctrl.n_probes, resolves=ctrl.n_resolves, recoveries=ctrl.n_stall_recoveries)
    rng = np.random.default_rng(31)
    knap = []
    cands, cm, budget = adaptive_setup(ref)
    for t in range(12):
        prof = SensitivityProfile(cands[-1], 0.9, tuple(cands))
        for L in range(ADAPTIVE_NL):
            for c in cands[:-1]:
                prof.alpha[(L, c)] = float(0.9 * np.exp(-rng.uniform(0.0, 3.0)))
        frac = float(rng.uniform(-0.1, 1.1))
        plan = allocate(prof, budget(frac), ADAPTIVE_CTX, 12, 64, ADAPTIVE_NL)
        knap.append(dict(alpha=[[L, cands.index(c), a] for (L, c), a in prof.alpha.items()], frac=frac,
                         plan=[cands.index(c) for c in plan]))
    probe = {}
    for resync in (1.0e-8, 2.0e-6):
        cands, cm, budget = adaptive_setup(ref, resync)
        ctrl = AdaptiveLayerController(cm, ADAPTIVE_NL, budget(0.6), cands, ctx_hint=ADAPTIVE_CTX, probe_prob=0.3,
                                       seed=1)
        probe[str(resync)] = [ctrl.effective_probe_prob(c) for c in (256, 4096, ADAPTIVE_CTX)]
    (HERE / "adaptive.json").write_text(json.dumps(dict(logs=logs, knapsack=knap, probe=probe)))


if __name__ == "__main__":
    main()
