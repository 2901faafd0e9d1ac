#!/usr/bin/env python
"""Benchmark of the self-speculative decode step (DRAFTKV) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--settle S] [--config c4|c3|c1|small]
                    [--impl draftkv|reference]
    python bench.py --kernel draft-attn|verify-attn|prefill-attn|gemm|gemm-layer [--batch B --ctx C --bits b
                    --keep f --T t --M m --K k --N n --iters i]     (one kernel alone)

A step is R (--rounds-per-step, default 10) draft / verify rounds over every
sequence of the batch; a round is gamma draft forwards over the compressed
cache, one (gamma+1)-token verify forward over the full cache, acceptance,
rollback and resync.  The default workload is configuration 4 of the
benchmark: Llama-3-8B shape (32 layers, 4096, 32q/8kv x 128, SwiGLU 14336,
vocab 128256), bf16 random-init N(0, 0.02) weights, context 32768, 4
sequences per GPU, greedy, (config, gamma) chosen per round by the Thompson
controller over the cost model instantiated with this GPU's measured HBM
bandwidth.  Inputs are synthetic (uniform token ids from seed 1 + rank);
weights are random (no checkpoints are available offline).

After the W warm-up steps, S further untimed rounds (default 60) let the
Thompson controller leave its flat prior: its exploration of arms that do not
pay is a transient of the first rounds of a long-running decode, not its
steady state.  The settle rounds are device-timed on their own and reported
under "explore"; the K timed steps measure the converged controller.  A
shorter run of rounds follows with per-launch CUDA events (kernel shares and
the GEMM roofline), then a leg that always drafts (the configuration's
first arm -- 8-bit keep 1 for the default set -- at gamma 2; "fixed_arm"),
so every run times drafting rounds whatever the controller chose.

Then the same prompts are decoded again from the start with gamma 0 (plain
full-KV decoding, no drafter cache): every token the speculative rounds
emitted is compared with it ("lossless", greedy output must be identical),
and its rounds at the positions of the timed region give the full-KV
baseline the speedup is measured against.

Multi-GPU (torchrun): sequences shard by rank (weak scaling, 4 per GPU);
the only collectives are the controller's inputs -- (accepted, context,
gamma) per sequence, gathered every 8 rounds by an asynchronous all-gather
and applied 2 rounds later on every rank, which keeps the replicated
controllers identical without holding the ranks in step every round -- and
one gather of the emitted token ids at the end.

The JSON line reports emitted tokens/s (value: device-timed rounds; e2e: wall
clock through the public engine API with its per-round host<->device copies),
the speedup over the GPU's own full-KV decode of the same sequences, that
speedup against CostModel.ceiling() of the benchmark's 4-bit keep-0.25 arm
(and of the arm the controller used most), the roofline of the dominant
kernel (the weight-streaming GEMM), the drafter / verify attention
bandwidth, clocks, and the numpy reference restatement (oracle/) timed on
the host cores at the BLAS library's default threads and at one thread.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "draft-kv_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

CONFIGS = {
    "c4": dict(preset="llama3-8b", ctx=32768, batch=4, temperature=0.0, gamma_max=8,
               workload="llama3-8b-shape bf16, ctx 32768, 4 seq/GPU, greedy, Thompson controller"),
    "c4f": dict(preset="llama3-8b", ctx=32768, batch=4, temperature=0.0, gamma_max=8, fixed=(8, 1.0, 2),
                workload="llama3-8b-shape bf16, ctx 32768, 4 seq/GPU, greedy, fixed 8b/keep1 gamma 2 (every round drafts)"),
    "c3": dict(preset="smollm2-135m", ctx=2048, batch=16, temperature=1.0, gamma_max=8,
               arms=[(8, 1.0), (4, 0.5), (4, 0.25), (2, 0.25)],
               workload="smollm2-135m-shape bf16, prompt 2048, 16 seq/GPU, T=1.0, 4-arm Thompson"),
    "c5": dict(preset="llama3-8b", ctx=262144, batch=1, temperature=0.0, gamma_max=8, arms=[(4, 0.25)],
               offload=True,
               workload="llama3-8b-shape bf16, ctx 262144, 1 seq/GPU, greedy; full KV in pinned host memory "
                        "(streamed over the host link by verify), int4 keep0.25 drafter in HBM"),
    "c1": dict(preset="distilgpt2", ctx=128, batch=1, temperature=0.0, gamma_max=4, fixed=(4, 1.0, 4),
               workload="distilgpt2-shape fp32, prompt 128, 1 seq, greedy, 4b/keep1 gamma 4"),
    "small": dict(preset=None, ctx=2048, batch=4, temperature=0.0, gamma_max=8,
                  workload="1.1B-class llama shape (8L/2048), ctx 2048, for quick checks"),
}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm_gbs=float(d["hbm_gbs"]), bf16_tflops=float(d["bf16_tflops"]), source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, source="fallback")


def model_config(name: str) -> dict:
    from draftkv import weights as W
    c = CONFIGS[name]
    if c["preset"]:
        return dict(W.PRESETS[c["preset"]])
    return W.llama_config(8, 2048, 16, 8, 5632, 32000, head_dim=128, theta=10000.0, tied=False, dtype="bf16")


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 50 ms) during the timed region.  start()
    returns once the sampler is live (its first line has arrived); only lines
    that arrive after the mark set at the start of the timed region count, so
    a short timed region still gets its own samples."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None
        self.mark = 0

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        t0 = time.perf_counter()
        while not self.lines and time.perf_counter() - t0 < 5.0:
            time.sleep(0.01)
        self.mark = len(self.lines)

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvidia-smi unavailable"])
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        during = self.lines[self.mark:] or self.lines[-1:]      # the last sample before, if none during
        for ln in during:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=mx, reasons=sorted(reasons),
                    samples=len(sm), during=len(self.lines) > self.mark)


def attention_split(ctx: int, ctx_max: int, pairs: int, sms: int = 148) -> int:
    """Keys per attention split for a run whose context grows from ctx to
    ctx_max with `pairs` (sequence, KV head) pairs: equal 64-key-aligned
    splits of ctx_max, as many as keep one wave of two CTAs per SM, when the
    pairs allow it; otherwise ctx / 8 as a power of two from 512 to 4096."""
    if pairs <= sms:
        n_split = max(1, (2 * sms) // pairs)
        return -(-ctx_max // (n_split * 64)) * 64
    split = 512
    while split * 2 <= min(4096, ctx // 8):
        split *= 2
    return split


# ---------------------------------------------------------------- CPU baseline
def _blas() -> dict:
    try:
        from threadpoolctl import threadpool_info
        info = [i for i in threadpool_info() if i.get("user_api") == "blas"]
    except Exception:       # noqa: BLE001 -- a missing helper must not sink the line
        info = []
    if not info:
        return dict(name="unknown", threads=os.cpu_count())
    return dict(name=f"{info[0].get('internal_api')} {info[0].get('version')}", threads=int(info[0]["num_threads"]))


def _oracle_model(cfg: dict, nl: int, block: np.ndarray):
    """The oracle (numpy restatement of the reference, pinned to it by the
    golden fixtures) for `cfg` cut to `nl` layers.  Weight values come from a
    fixed random block: timing does not depend on them and this keeps set-up
    short."""
    import oracle
    from draftkv import weights as W

    def fill(shape):
        n = int(np.prod(shape))
        return np.resize(block, n).reshape(shape).astype(np.float32)

    cc = dict(cfg)
    key = "num_hidden_layers" if "num_hidden_layers" in cc else "n_layer"
    cc[key] = nl
    if cc["arch"] != "llama":
        return oracle.OracleModel(W.make_weights(cc, seed=0, std=0.02), cc)
    d, H, KV = cc["hidden_size"], cc["num_attention_heads"], cc["num_key_value_heads"]
    D, F, V = cc.get("head_dim") or d // H, cc["intermediate_size"], cc["vocab_size"]
    shapes = {"model.embed_tokens.weight": (V, d), "model.norm.weight": None}
    for i in range(nl):
        p = f"model.layers.{i}."
        shapes.update({p + "self_attn.q_proj.weight": (H * D, d), p + "self_attn.k_proj.weight": (KV * D, d),
                       p + "self_attn.v_proj.weight": (KV * D, d), p + "self_attn.o_proj.weight": (d, H * D),
                       p + "mlp.gate_proj.weight": (F, d), p + "mlp.up_proj.weight": (F, d),
                       p + "mlp.down_proj.weight": (d, F), p + "input_layernorm.weight": None,
                       p + "post_attention_layernorm.weight": None})
    if not cc.get("tie_word_embeddings", True):
        shapes["lm_head.weight"] = (V, d)
    return oracle.OracleModel({k: (fill(s) if s else np.ones(d, np.float32)) for k, s in shapes.items()}, cc)


def _oracle_full(m, ctx: int, block: np.ndarray):
    import oracle
    f = oracle.OracleFull(m.n_layers)
    kblk = np.resize(block, (ctx * m.n_kv_heads * m.d_head)).reshape(ctx, m.n_kv_heads, m.d_head)
    for L in range(m.n_layers):
        f.rows[L] = [(kblk[i].astype(np.float64), kblk[i], i) for i in range(ctx)]
    return f


def oracle_forward_costs(cfg: dict, ctx: int, gamma: int, bits: int, keep: float) -> dict:
    """Seconds of the oracle's three forwards of one sequence at context ctx:
    verify (gamma+1 tokens over the full cache), baseline (1 token over the
    full cache) and draft (1 token over the compressed cache of `bits`/`keep`),
    for the whole model: timed on 0- and 2-layer models of the same shape and
    extrapolated linearly in the layer count (the per-layer work is identical)."""
    import oracle
    from draftkv.config import CompressionConfig

    full_layers = cfg["num_hidden_layers"] if "num_hidden_layers" in cfg else cfg["n_layer"]
    block = (np.random.default_rng(0).standard_normal(1 << 20) * 0.02).astype(np.float32)
    cc = CompressionConfig(bits, keep)
    res = {}
    for nl in (0, 2):
        m = _oracle_model(cfg, nl, block)
        f = _oracle_full(m, ctx, block)
        comp = oracle.OracleComp(m.n_layers, cc)
        if nl:
            comp.sync_from(f, 0)
        toks = np.arange(gamma + 1) % m.vocab_size
        t0 = time.perf_counter()
        m.forward(toks, f, ctx)
        tv = time.perf_counter() - t0
        f.truncate(ctx)
        t0 = time.perf_counter()
        m.forward(toks[:1], f, ctx)
        tb = time.perf_counter() - t0
        f.truncate(ctx)
        comp.seen = max(comp.seen, ctx)
        t0 = time.perf_counter()
        m.forward(toks[:1], comp, ctx)
        td = time.perf_counter() - t0
        res[nl] = (tv, tb, td)
        del m, f, comp
    per_layer = [(res[2][i] - res[0][i]) / 2 for i in range(3)]
    tv, tb, td = [res[0][i] + full_layers * per_layer[i] for i in range(3)]
    return dict(verify_s=tv, baseline_s=tb, draft_s=td, layers=full_layers)


def cpu_baseline(cfg: dict, ctx: int, mean_gamma: float, tokens_per_round: float, bits: int, keep: float) -> dict:
    """The oracle timed on this host's cores on a bounded sample of the GPU
    run's own workload: one sequence's forwards at the same context,
    extrapolated to the full layer count, at the GPU run's measured
    per-sequence tokens per round, mean gamma and most used drafter arm (the
    reference engine is batch-1: its sequences run one after another, so its
    tokens/s is that of one sequence).  Taken at the BLAS library's default
    thread count (the value) and at one thread."""
    from threadpoolctl import threadpool_limits

    t_start = time.perf_counter()
    blas = _blas()
    g = max(1, int(round(mean_gamma)))

    def rate(c):
        spec = tokens_per_round / (mean_gamma * c["draft_s"] + c["verify_s"]) if mean_gamma > 0 else None
        return spec, 1.0 / c["baseline_s"]

    c_def = oracle_forward_costs(cfg, ctx, g, bits, keep)
    with threadpool_limits(limits=1, user_api="blas"):
        c_one = oracle_forward_costs(cfg, ctx, g, bits, keep)
    spec_d, base_d = rate(c_def)
    spec_1, base_1 = rate(c_one)
    value = spec_d if spec_d is not None else base_d
    return dict(value=round(value, 5), unit="tokens/s", cores=blas["threads"], kind="port",
                blas=blas["name"], host_cpus=os.cpu_count(),
                speculative_tps=None if spec_d is None else round(spec_d, 5), baseline_decode_tps=round(base_d, 5),
                one_thread={"speculative_tps": None if spec_1 is None else round(spec_1, 5),
                            "baseline_decode_tps": round(base_1, 5)},
                forward_s={"verify": round(c_def["verify_s"], 3), "baseline": round(c_def["baseline_s"], 3),
                           "draft": round(c_def["draft_s"], 3)},
                sample=(f"oracle (numpy restatement of the reference, pinned to it) forwards of 0- and 2-layer "
                        f"models of this shape at ctx {ctx}, 1 sequence, extrapolated to {c_def['layers']} layers "
                        f"(extrapolated); speculative rate at the GPU run's measured {tokens_per_round:.3f} "
                        f"tokens/round per sequence, mean gamma {mean_gamma:.2f} (verify timed at gamma {g}), "
                        f"drafter {bits}b/keep{keep:g}; BLAS threads {blas['threads']} (value) and 1"),
                seconds=round(time.perf_counter() - t_start, 1))


# ---------------------------------------------------------------- GPU run
def json_stdout():
    """A private handle on the process's real stdout for the one JSON line;
    file descriptor 1 itself is pointed at stderr, so anything else written
    there (a communication library's banner, say) cannot join the line."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    out = json_stdout()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    from draftkv import (CompressionConfig, CostModel, DraftKVEngine, FixedPolicy, ThompsonController,
                         default_arms, from_config)
    from draftkv import _lib
    from draftkv.models import random_device_weights

    conf = CONFIGS[args.config]
    cfg = model_config(args.config)
    ctx = args.ctx or conf["ctx"]
    B = args.batch or conf["batch"]
    T = conf["temperature"]
    G = conf["gamma_max"]
    R = args.rounds_per_step
    pk = peaks()
    t_setup = time.perf_counter()
    wts = random_device_weights(cfg, seed=0, std=0.02)
    # controller settle: untimed rounds after the warm-up in which the
    # Thompson controller explores its arms (its posterior starts flat); the
    # timed rounds then measure the steady state it converges to.  The settle
    # rounds are timed on their own and reported as "explore".
    settle = 0 if "fixed" in conf else args.settle
    timed_n = args.steps * R
    prof_n = min(timed_n, args.prof_rounds)
    fixed_n = 0 if ("fixed" in conf or args.no_fixed_arm) else min(timed_n, args.fixed_rounds)
    spec_rounds = args.warmup * R + settle + timed_n + prof_n + fixed_n + 8      # + calibration rounds
    max_new = spec_rounds * (G + 1) + 8
    # keys per attention split: fixed for the model for the whole run (verify
    # and decode rows then share split boundaries).  When the (sequence, KV
    # head) pairs fit two CTAs per SM, the run's longest context is cut into
    # as many equal 64-key-aligned splits as keep one wave of two CTAs per
    # SM (measured on B200, batch 4 at ctx 33600: 3776-key splits 129 us
    # against 135 us for 4096-key ones, whose last split is nearly empty);
    # otherwise ctx / 8, a power of two from 512 to 4096, keeps 8 splits per
    # pair in flight while each streams long enough to amortise its merge.
    n_kv_heads = cfg.get("num_key_value_heads", cfg.get("n_head", 1))
    pairs = B * n_kv_heads
    split = args.split_keys or attention_split(ctx, ctx + max_new, pairs)
    model = from_config(wts, cfg, split_keys=split)
    del wts
    torch.cuda.empty_cache()
    n_kv = model.n_kv_heads
    h2d_bw = None
    if conf.get("offload"):
        # the full cache is read over the host link: measure it (pinned -> device)
        hbuf = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
        dbuf = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
        dbuf.copy_(hbuf, non_blocking=True)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(3):
            dbuf.copy_(hbuf, non_blocking=True)
        torch.cuda.synchronize()
        h2d_bw = 3 * (1 << 30) / (time.perf_counter() - t0)
        del hbuf, dbuf
    cm = CostModel(n_layers=model.n_layers, n_kv_heads=n_kv, d_head=model.d_head, weight_bytes=float(model.weight_bytes),
                   bandwidth=pk["hbm_gbs"] * 1e9, batch=B, **({"full_kv_bandwidth": h2d_bw} if h2d_bw else {}))
    # the arm the calibration rounds and the always-drafting leg use: the
    # first of the configuration's arms (8-bit keep 1 for the default set)
    lead_cfg = CompressionConfig(*conf["arms"][0]) if "arms" in conf else CompressionConfig(8, 1.0)
    if "fixed" in conf:
        b_, k_, g_ = conf["fixed"]
        ctrl = FixedPolicy(CompressionConfig(b_, k_), g_)
    else:
        arms = [CompressionConfig(b, k) for b, k in conf["arms"]] if "arms" in conf else default_arms()
        ctrl = ThompsonController(cm, arms, gamma_max=G, seed=0)

    exchange = None
    if world > 1:
        # the controller's inputs cross ranks in batches of 8 rounds, applied
        # 2 rounds after they ship (asynchronous NCCL all-gather)
        from draftkv.dist import ControllerExchange
        exchange = ControllerExchange(B, period=8, lag=2, device="cuda")

    engine = DraftKVEngine(model, ctrl, seed=rank, gamma_max=G)
    engine.offload_full = bool(conf.get("offload"))
    vocab = model.vocab_size
    prompts = [[int(x) for x in np.random.default_rng(1 + 1000 * rank + b).integers(0, vocab, ctx)] for b in range(B)]
    torch.cuda.synchronize()
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record()
    sess = engine.session(prompts, max_new, T, exchange=exchange)        # the prefill
    p1.record()
    torch.cuda.synchronize()
    prefill = {"tokens": B * (ctx - 1), "seconds": round(p0.elapsed_time(p1) / 1e3, 3),
               "tokens_per_s": round(B * (ctx - 1) / (p0.elapsed_time(p1) / 1e3), 1),
               "basis": "engine.session(): chunked full-cache forwards of max(512, 2048 / batch) tokens a sequence, no logits; "
                        "CUDA events (includes the host's launch of the chunks)"}
    setup_s = time.perf_counter() - t_setup

    for _ in range(args.warmup * R):
        sess.round()
    # CostModel constants measured on this device (a few real rounds at a
    # fixed arm, part of the warm-up), then the controller built on them; the
    # constants are averaged over ranks so replicated controllers stay equal
    calib = None
    if "fixed" not in conf and not args.no_calibrate:
        from draftkv.calibrate import calibrate_cost_model
        cm_cal, calib = calibrate_cost_model(sess, cm, lead_cfg, 2)
        if world > 1:
            v = torch.tensor([cm_cal.bandwidth, cm_cal.full_kv_bandwidth, cm_cal.fixed_draft, cm_cal.fixed_verify,
                              cm_cal.resync_per_token, cm_cal.rebuild_per_token or 0.0], dtype=torch.float64,
                             device="cuda")
            dist.all_reduce(v, op=dist.ReduceOp.SUM)
            v = (v / world).tolist()
            from dataclasses import replace
            cm_cal = replace(cm_cal, bandwidth=v[0], full_kv_bandwidth=v[1], fixed_draft=v[2], fixed_verify=v[3],
                             resync_per_token=v[4], rebuild_per_token=v[5] or None)
        arms = [CompressionConfig(b, k) for b, k in conf["arms"]] if "arms" in conf else default_arms()
        ctrl = ThompsonController(cm_cal, arms, gamma_max=G, seed=0)
        engine.controller = ctrl
        calib = {k: (round(v, 9) if isinstance(v, float) else v) for k, v in calib.items()}
        calib.update({"used": {"bandwidth": cm_cal.bandwidth, "full_kv_bandwidth": cm_cal.full_kv_bandwidth,
                               "fixed_draft": cm_cal.fixed_draft, "fixed_verify": cm_cal.fixed_verify,
                               "resync_per_token": cm_cal.resync_per_token,
                               "rebuild_per_token": cm_cal.rebuild_per_token},
                      "defaults": {"bandwidth": cm.bandwidth, "fixed_draft": cm.fixed_draft,
                                   "fixed_verify": cm.fixed_verify, "resync_per_token": cm.resync_per_token},
                      "ceiling_4b_keep0.25": round(cm_cal.ceiling(CompressionConfig(4, 0.25), ctx), 4)})
    explore = None
    if settle:
        torch.cuda.synchronize()
        x0 = torch.cuda.Event(enable_timing=True)
        x1 = torch.cuda.Event(enable_timing=True)
        x0.record()
        xtoks = 0
        for _ in range(settle):
            sess.round()
            _c, g_r, o = sess.last
            xtoks += sum(1 + kk for kk, _e in o) if g_r > 0 else len(o)
        x1.record()
        torch.cuda.synchronize()
        explore = {"rounds": settle, "tokens": xtoks, "device_s": x0.elapsed_time(x1) / 1e3}

    def kept_of(c_, n):
        return min(n, max(c_.sink + c_.recent, int(round(c_.keep_frac * n))))

    def timed_rounds(s_, k, profile):
        """k rounds of session s_ between barriers and synchronizes, device
        timed with CUDA events on the launching stream; nvidia-smi samples
        the clocks meanwhile."""
        toks = 0
        cfgs = {}
        gammas = []
        dbytes = 0.0       # algorithmic drafter-attention bytes of the rounds (per config used)
        # the clock sampler is live before the barrier, so every rank enters
        # the timed region together
        clk = ClockSampler(local)
        clk.start()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        if profile:
            _lib.call("dkv_prof_start", 400000)
        clk.mark = len(clk.lines)
        t0 = time.perf_counter()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if profile:
            torch.cuda.cudart().cudaProfilerStart()     # ncu --profile-from-start off captures this range
        e0.record()
        for _ in range(k):
            s_.round()
            cfg_r, g_r, o = s_.last
            toks += sum(1 + kk for kk, _e in o) if g_r > 0 else len(o)
            cfgs[cfg_r] = cfgs.get(cfg_r, 0) + 1
            gammas.append(g_r)
            if g_r > 0:
                dbytes += (g_r * model.n_layers * B * n_kv * kept_of(cfg_r, ctx) * 2
                           * cfg_r.bytes_per_entry(model.d_head))
        e1.record()
        if profile:
            torch.cuda.cudart().cudaProfilerStop()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        if world > 1:
            dist.barrier()
        clocks = clk.stop()
        if profile:
            _lib.call("dkv_prof_stop")
        dev_ms = e0.elapsed_time(e1)
        return toks, dev_ms / 1e3, wall, clocks, cfgs, gammas, dbytes

    # the headline: K steps of R rounds with no per-launch events; then a
    # shorter run of rounds with per-launch CUDA events for the kernel roofline
    start_len = [len(t) for t in sess.toks]
    toks, dev_s, wall_s, clocks, cfg_counts, gammas, _ = timed_rounds(sess, timed_n, profile=False)
    timed_emit = [len(t) - n for t, n in zip(sess.toks, start_len)]
    _, prof_dev_s, _, _, _, _, d_bytes = timed_rounds(sess, prof_n, profile=True)
    prof = {}
    import ctypes as C
    lib = _lib.load()
    names = ["gemm", "attn_full", "attn_comp", "append", "rebuild", "norm", "embed", "sample", "accept"]
    for i, nm in enumerate(names):
        ms, n, by = C.c_double(), C.c_int64(), C.c_double()
        _lib.check(lib.dkv_prof_summary(i, C.byref(ms), C.byref(n), C.byref(by)), "dkv_prof_summary")
        prof[nm] = dict(ms=ms.value, launches=n.value, bytes=by.value)
    prof_launches = sum(v["launches"] for v in prof.values())
    # a leg that always drafts: the 8-bit keep-1 arm at gamma 2 (the arm whose
    # acceptance random weights leave high), so that every run, at every N,
    # times drafting rounds whatever the controller chose
    fixed_leg = None
    if fixed_n:
        saved_ctrl = engine.controller
        engine.controller = FixedPolicy(lead_cfg, 2)
        sess.round()                              # the drafter cache switches to the arm
        f_start = [len(t) for t in sess.toks]
        ftoks, fdev_s, _, _, _, _, _ = timed_rounds(sess, fixed_n, profile=False)
        engine.controller = saved_ctrl
        fixed_leg = dict(tokens=ftoks, dev_s=fdev_s,
                         tpr=sum(len(t) - n for t, n in zip(sess.toks, f_start)) / max(1, fixed_n) / B)
    sess.finish()
    spec_streams = [list(t) for t in sess.toks]
    plen = len(prompts[0])
    gathered = None
    if world > 1:
        from draftkv.dist import gather_tokens
        gathered = sum(len(t) - plen for t in gather_tokens(spec_streams))
    del sess
    model._graphs.clear()
    torch.cuda.empty_cache()

    # Full-KV decode (gamma 0, no drafter cache) of the same prompts from the
    # start: it replays every token the speculative rounds emitted
    # (losslessness: greedy output must be identical) and its rounds at the
    # positions of the timed region are the full-KV baseline.
    def agree(v, op):
        if world == 1:
            return v
        t_ = torch.tensor([v], dtype=torch.int64, device="cuda")
        dist.all_reduce(t_, op=op)
        return int(t_.item())

    n_check = agree(max(len(t) - plen for t in spec_streams), dist.ReduceOp.MAX if world > 1 else None)
    b_start = agree(min(start_len) - plen, dist.ReduceOp.MIN if world > 1 else None)
    b_len = agree(max(1, int(round(float(np.mean(timed_emit))))), dist.ReduceOp.MAX if world > 1 else None)
    b_len = min(b_len, n_check - b_start)
    beng = DraftKVEngine(model, FixedPolicy(CompressionConfig(16, 1.0), 0), seed=rank, gamma_max=G)
    beng.offload_full = bool(conf.get("offload"))
    # a fixed policy needs no replication: ranks decode independently
    bsess = beng.session(prompts, n_check, T)
    for _ in range(b_start):
        bsess.round()
    btoks, bdev_s, bwall_s, _, _, _, _ = timed_rounds(bsess, b_len, profile=False)
    while not bsess.done:
        bsess.round()
    compared = 0
    lossless = True
    for a_, b_ in zip(spec_streams, bsess.toks):
        n_ = min(len(a_), len(b_))
        compared += n_ - plen
        lossless = lossless and a_[:n_] == b_[:n_]
    lossless = bool(agree(1 if lossless else 0, dist.ReduceOp.MIN if world > 1 else None))
    compared = agree(compared, dist.ReduceOp.SUM if world > 1 else None)
    del bsess
    model._graphs.clear()
    chain = gemm_decode_chain(model, B, pk) if model.dtype == _lib.BF16 else None

    # reduce over ranks: max time, summed tokens
    vals = torch.tensor([toks, dev_s, wall_s, btoks, bdev_s], dtype=torch.float64, device="cuda")
    if world > 1:
        tot = vals.clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        toks_all, btoks_all = tot[0].item(), tot[3].item()
        dev_s, wall_s, bdev_s = mx[1].item(), mx[2].item(), mx[4].item()
    else:
        toks_all, btoks_all = toks, btoks
    value = toks_all / dev_s
    e2e = toks_all / wall_s
    if explore is not None:
        xv = torch.tensor([explore["tokens"], explore["device_s"]], dtype=torch.float64, device="cuda")
        if world > 1:
            xs = xv.clone()
            dist.all_reduce(xs, op=dist.ReduceOp.SUM)
            xm = xv.clone()
            dist.all_reduce(xm, op=dist.ReduceOp.MAX)
            xv = torch.stack([xs[0], xm[1]])
        explore["tokens_per_s"] = round(xv[0].item() / xv[1].item(), 3)
    base_tps = btoks_all / bdev_s
    speedup = value / base_tps
    fixed_line = None
    if fixed_leg is not None:
        fv = torch.tensor([fixed_leg["tokens"], fixed_leg["dev_s"]], dtype=torch.float64, device="cuda")
        if world > 1:
            fs = fv.clone()
            dist.all_reduce(fs, op=dist.ReduceOp.SUM)
            fm = fv.clone()
            dist.all_reduce(fm, op=dist.ReduceOp.MAX)
            fv = torch.stack([fs[0], fm[1]])
        ftps = fv[0].item() / fv[1].item()
        fixed_line = {"cfg": lead_cfg.label(), "gamma": 2, "rounds": fixed_n, "tokens_per_s": round(ftps, 3),
                      "speedup_vs_full_kv": round(ftps / base_tps, 4),
                      "tokens_per_round_per_seq": round(fixed_leg["tpr"], 3)}
    top_cfg = max(cfg_counts.items(), key=lambda kv: kv[1])[0] if cfg_counts else CompressionConfig(4, 0.25)
    # the benchmark's target is stated against the 4-bit keep-0.25 arm's ceiling
    target_cfg = CompressionConfig(4, 0.25)
    ceiling = cm.ceiling(target_cfg, ctx)
    arm_ceiling = cm.ceiling(top_cfg, ctx)
    mean_gamma = float(np.mean(gammas)) if gammas else 0.0
    tpr = toks / max(1, timed_n) / B

    # roofline: dominant kernel = the weight-streaming GEMM
    g = prof["gemm"]
    gemm_gbs = g["bytes"] / (g["ms"] / 1e3) / 1e9 if g["ms"] > 0 else 0.0
    bytes_per_launch = g["bytes"] / max(1, g["launches"])
    kv_elem = 2 if model.dtype == _lib.BF16 else 4
    # attention bandwidth from algorithmic bytes of the launches in the profiled rounds
    v_bytes = prof_n * model.n_layers * B * n_kv * ctx * 2 * model.d_head * kv_elem
    a_draft_gbs = d_bytes / (prof["attn_comp"]["ms"] / 1e3) / 1e9 if prof["attn_comp"]["ms"] > 0 else None
    a_full_gbs = v_bytes / (prof["attn_full"]["ms"] / 1e3) / 1e9 if prof["attn_full"]["ms"] > 0 else None
    ratio = gemm_traffic_ratio()
    traffic = round(bytes_per_launch * ratio["ratio"]) if ratio else None
    kernel_share = {k: round(v["ms"] / max(1e-9, sum(x["ms"] for x in prof.values())), 4) for k, v in prof.items()
                    if v["launches"]}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            cpu = cpu_baseline(cfg, ctx, mean_gamma, tpr, top_cfg.bits, top_cfg.keep_frac)
        except Exception as e:  # noqa: BLE001 -- the CPU leg must not sink the GPU line
            cpu = dict(value=None, unit="tokens/s", cores=os.cpu_count(), kind="port", sample=f"failed: {e}")

    h2d = B * 4 + (G + 2) * 8
    d2h = B * 4 + B * (G + 2) * 4
    line = {
        "metric": "emitted tokens/s (box), speedup vs full-KV decode vs ceiling; attn HBM GB/s",
        "value": round(value, 3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_s / args.steps * 1e3, 3),
        "rounds_per_step": R,
        "ms_per_round": round(dev_s / timed_n * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if model.dtype == _lib.BF16 else "f32",
        "data": "synthetic (uniform token ids; random-init N(0,0.02) weights)",
        "config": {"workload": conf["workload"], "ctx": ctx, "seqs_per_gpu": B, "global_seqs": B * world,
                   "attn_split_keys": split, "temperature": T, "gamma_max": G,
                   "arms": len(getattr(ctrl, "arms", [1])),
                   "step": f"{R} draft/verify rounds of every sequence",
                   "parallelism": f"dp{world} (sequences sharded by rank)",
                   "l2": f"inputs > L2 (weights {model.weight_bytes / 1e9:.1f} GB + full KV "
                         f"{B * model.n_layers * 2 * n_kv * model.d_head * 2 * ctx / 1e9:.1f} GB stream every round)",
                   "full_kv": "pinned host memory" if conf.get("offload") else "HBM",
                   **({"h2d_gbs": round(h2d_bw / 1e9, 1)} if h2d_bw else {})},
        # token identity holds for greedy decoding; with sampling the two
        # decodes draw different random numbers and agree in distribution only
        # (the first-token TV test of the GPU tests checks that)
        "lossless": lossless if T == 0.0 else None,
        "lossless_tokens_compared": compared if T == 0.0 else 0,
        "tokens_gathered": gathered,
        "exchange": (f"batched async all-gather: every {exchange.period} rounds, applied {exchange.lag} rounds later, "
                     f"{exchange.batches} batches" if exchange is not None else None),
        "cost_model_calibration": calib,
        "fixed_arm": fixed_line,
        "controller_settle_rounds": settle,
        "explore": ({"rounds": explore["rounds"], "tokens_per_s": explore["tokens_per_s"],
                     "speedup_vs_full_kv": round(explore["tokens_per_s"] / base_tps, 4)} if explore else None),
        "speedup_vs_full_kv": round(speedup, 4),
        "full_kv_decode_tps": round(base_tps, 3),
        "full_kv_decode_tps_per_gpu": round(base_tps / world, 3),
        "full_kv_rounds_timed": b_len,
        "ceiling": round(ceiling, 4),
        "ceiling_cfg": target_cfg.label(),
        "speedup_frac_of_ceiling": round(speedup / ceiling, 4) if ceiling else None,
        "arm_ceiling": round(arm_ceiling, 4),
        "arm_ceiling_cfg": top_cfg.label(),
        "speedup_frac_of_arm_ceiling": round(speedup / arm_ceiling, 4) if arm_ceiling else None,
        "mean_gamma": round(mean_gamma, 3),
        "tokens_per_round_per_seq": round(tpr, 3),
        "cfg_rounds": {c.label(): n for c, n in cfg_counts.items()},
        "attn_draft_gbs": round(a_draft_gbs, 1) if a_draft_gbs else None,
        "attn_verify_gbs": round(a_full_gbs, 1) if a_full_gbs else None,
        "roofline": {"bound": "hbm", "kernel": "gemm (weight streaming)", "achieved": round(gemm_gbs, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(gemm_gbs / pk["hbm_gbs"], 4),
                     "peak_source": pk["source"], "traffic": traffic,
                     "traffic_basis": ratio["basis"] if ratio else None,
                     "bytes_per_launch": round(bytes_per_launch),
                     "avg_launch_us": round(g["ms"] * 1e3 / max(1, g["launches"]), 2),
                     "rounds_profiled": prof_n,
                     "decode_chain": chain},
        "kernel_time_share": kernel_share,
        "gpu_launches": int(round(prof_launches / max(1, prof_n) * timed_n)),
        "gpu_launches_basis": f"{prof_launches} launches counted over {prof_n} profiled rounds, scaled to "
                              f"the {timed_n} timed rounds",
        "clocks": clocks,
        "e2e": {"value": round(e2e, 3), "unit": "tokens/s", "h2d_bytes_per_step": h2d * R,
                "d2h_bytes_per_step": d2h * R},
        "cpu_baseline": cpu,
        "setup_s": round(setup_s, 1),
        "prefill": prefill,
    }
    if rank == 0:
        print(json.dumps(line), file=out, flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def gemm_traffic_ratio() -> dict | None:
    """DRAM bytes per algorithmic byte of the weight GEMM, from the committed
    ncu summary (a line `traffic_ratio: <x>` in profiles/gemm_traffic_*.md,
    measured over every GEMM launch of a captured decode round); the bench
    scales its live algorithmic bytes per launch by it."""
    import re
    for f in sorted((ROOT / "profiles").glob("gemm_traffic_*.md")):
        m = re.search(r"^traffic_ratio:\s*([0-9.]+)", f.read_text(), re.M)
        if m:
            return dict(ratio=float(m.group(1)), basis=f"profiles/{f.name}: ncu dram__bytes over algorithmic bytes")
    return None


def run_reference(args) -> None:
    """The reference's own CPU algorithm (the oracle: a numpy restatement of
    it, pinned to outputs of the reference by the golden fixtures) on this
    host's cores with the BLAS library's default threads.  A step is one
    timed forward of a one-layer model of the configuration's shape for one
    token of one sequence over a full cache at the configuration's context;
    the embedding + head part is timed on a zero-layer model, and the value
    is the full-KV decode rate of the whole model (that part plus n_layers x
    the per-layer part): the reference decodes its sequences one after
    another, and its full-KV decode needs no acceptance figure.  The draft
    and verify forwards of the benchmark's 4-bit keep-0.25 arm are timed
    once beside it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    conf = CONFIGS[args.config]
    cfg = model_config(args.config)
    ctx = args.ctx or conf["ctx"]
    n_layers = cfg["num_hidden_layers"] if "num_hidden_layers" in cfg else cfg["n_layer"]
    bits, keep, gamma = conf.get("fixed", (4, 0.25, 4))
    t_start = time.perf_counter()
    blas = _blas()
    block = (np.random.default_rng(0).standard_normal(1 << 20) * 0.02).astype(np.float32)
    m0 = _oracle_model(cfg, 0, block)
    f0 = _oracle_full(m0, ctx, block)
    m1 = _oracle_model(cfg, 1, block)
    f1 = _oracle_full(m1, ctx, block)
    tok = np.array([1])

    def step(m, f):
        t0 = time.perf_counter()
        m.forward(tok, f, ctx)
        dt = time.perf_counter() - t0
        f.truncate(ctx)
        return dt

    t_rest = statistics.median(step(m0, f0) for _ in range(3))
    for _ in range(args.warmup):
        step(m1, f1)
    times = [step(m1, f1) for _ in range(args.steps)]
    t_layer = max(1e-9, statistics.median(times) - t_rest)
    t_token = t_rest + n_layers * t_layer
    value = 1.0 / t_token
    timed_s = sum(times)
    spec = None
    try:
        c = oracle_forward_costs(cfg, ctx, gamma, bits, keep)
        spec = {"arm": f"{bits}b/keep{keep:g}", "gamma": gamma, "forward_s": {
                    "verify": round(c["verify_s"], 3), "draft": round(c["draft_s"], 3),
                    "baseline": round(c["baseline_s"], 3)},
                "speculative_tps_if_every_draft_accepted": round((gamma + 1) / (gamma * c["draft_s"] + c["verify_s"]), 5)}
    except Exception as e:  # noqa: BLE001 -- the bracket must not sink the line
        spec = {"failed": str(e)}
    cpu = dict(value=round(value, 5), unit="tokens/s", cores=blas["threads"], kind="port", blas=blas["name"],
               host_cpus=os.cpu_count(),
               sample=(f"oracle one-layer forwards (1 token, 1 sequence, full cache at ctx {ctx}), {args.steps} "
                       f"timed steps of {statistics.median(times):.3f} s; zero-layer forward {t_rest:.3f} s; "
                       f"full-KV decode rate of {n_layers} layers extrapolated"))
    line = {
        "impl": "reference",
        "metric": "emitted tokens/s (box), speedup vs full-KV decode vs ceiling; attn HBM GB/s",
        "value": cpu["value"], "unit": "tokens/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(statistics.mean(times) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (numpy reference)",
        "data": "synthetic", "config": {"workload": conf["workload"], "ctx": ctx,
                                        "step": "one forward of a one-layer model (1 token, 1 sequence)"},
        "reference_mode": "full-KV decode (generate_baseline) of one sequence at a time",
        "per_layer_s": round(t_layer, 4), "per_token_s": round(t_token, 3),
        "speculative_bracket": spec,
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "timed_s": round(timed_s, 2),
        "wall_s": round(time.perf_counter() - t_start, 1),
    }
    print(json.dumps(line), flush=True)


def gemm_decode_chain(model, N: int, pk: dict) -> dict:
    """The weight GEMMs of one decode forward (every layer's QKV, O, gate/up,
    down and the head, with the model's packed weights) back to back as the
    forward launches them -- programmatic dependent launch, one CUDA graph --
    at N tokens, store epilogues into scratch.  Device time of the graph over
    the weights' bytes: the weight stream's rate with launches overlapped,
    beside the per-launch CUDA-event figure of the profiled rounds (whose
    event between every two launches serialises them)."""
    import ctypes as C
    import torch
    from draftkv import _lib

    dm, HD, KD, dff = model.d_model, model.n_heads * model.d_head, model.n_kv_heads * model.d_head, model.d_ff

    def r128(x):
        return (x + 127) // 128 * 128

    shapes = {"w_qkv": (r128(HD + 2 * KD), dm), "w_o": (r128(dm), HD), "w_up": (r128(2 * dff), dm),
              "w_down": (r128(dm), dff)}
    seq = [(ly[k], *shapes[k]) for ly in model._keep[5] for k in ("w_qkv", "w_o", "w_up", "w_down")]
    seq.append((model._keep[2], model.vocab_pad, dm))
    g = torch.Generator(device="cuda").manual_seed(3)
    xs = {K: torch.randn((N, K), generator=g, device="cuda").to(torch.bfloat16) for _, _, K in seq}
    outs = {M: torch.zeros((N, M), dtype=torch.float32, device="cuda") for _, M, _ in seq}
    work = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    epis = []
    for _, M, K in seq:
        e = _lib.EpilogueS()
        e.kind = _lib.EPI_STORE
        e.out_f32 = outs[M].data_ptr()
        e.ld_out = M
        e.act_dtype = _lib.BF16
        epis.append(e)

    def run():
        for (w, M, K), e in zip(seq, epis):
            _lib.call("dkv_gemm", xs[K].data_ptr(), _lib.BF16, w.data_ptr(), _lib.BF16, M, N, K, C.byref(e),
                      work.data_ptr(), work.numel(), _lib.stream_ptr())

    run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    for _ in range(3):
        graph.replay()
    ts = []
    for _ in range(5):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ms = statistics.median(ts)
    by = sum(M * K * 2 + N * K * 2 + N * M * 4 for _, M, K in seq)
    gbs = by / (ms / 1e3) / 1e9
    del graph
    return {"tokens": N, "launches": len(seq), "ms_per_forward": round(ms, 3), "bytes_per_forward": int(by),
            "achieved": round(gbs, 1), "frac": round(gbs / pk["hbm_gbs"], 4),
            "basis": "the forward's weight GEMMs back to back in one CUDA graph (PDL), device time"}


def run_kernel(args) -> None:
    """One hot-path kernel alone on a seeded synthetic case (for roofline and
    ncu captures), one JSON line.  Inputs exceed L2 (126 MB) and L2 is
    flushed between timed launches.

      draft-attn   drafter attention (configuration 2 shape by default:
                   batch 32, ctx 32768, 8 kv x 128, group 4, int4 keep 0.25)
      verify-attn  full-cache attention for T query tokens per sequence
      prefill-attn the same for a prompt chunk (T = 512 tokens at the end of
                   the context, pages in the block pool's allocation order,
                   16384-key splits): the tcgen05 prefill kernel, in TF/s
      gemm         weight-streaming GEMM, M x K weights, N tokens
      gemm-layer   the four projections of a decoder layer (Llama-3-8B shape:
                   QKV, O, gate/up, down) back to back as the forward launches
                   them (programmatic dependent launch, one CUDA graph), over
                   8 layers of distinct weights (3.5 GB: inputs far larger than
                   L2, no flush); per-layer time = graph time / 8
    """
    import torch
    from draftkv import _lib, FullKVCache, CompressedKVCache, CompressionConfig
    import ctypes as C
    _lib.load()
    pk = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    iters = args.iters

    def timeit(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(iters):
            flush.zero_()
            # ~50 us of device time so that the host has queued the launch
            # before the first event fires: the events then bracket device
            # time only, not the host's submission latency
            torch.cuda._sleep(100_000)
            a = torch.cuda.Event(enable_timing=True)
            b_ = torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b_.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b_) * 1e3)
        return statistics.median(ts)

    B = args.batch or (32 if args.kernel == "draft-attn" else 4)
    ctx = args.ctx or 32768
    n_kv, d, G = 8, 128, 4
    line = {"kernel": args.kernel}

    def full_cache():
        full = FullKVCache(1, n_kv, d, "bf16", capacity=ctx + 64, batch=B)
        for b in range(B):
            full.ensure(b, ctx + 16)
        if not (args.no_shuffle or args.kernel == "prefill-attn"):
            # configuration 2: the page table shuffled from a seed (pages of a
            # sequence scattered over the pool)
            used = sorted({blk for b in range(B) for blk in full.block_tables[b][0]})
            perm = dict(zip(used, np.random.default_rng(7).permutation(used).tolist()))
            for b in range(B):
                tbl = full.block_tables[b][0]
                for i, blk in enumerate(tbl):
                    tbl[i] = perm[blk]
                    full.table_host[b, 0, i] = perm[blk]
            full._dirty = True
        g = torch.Generator(device="cuda").manual_seed(0)
        # K/V ~ N(0, 1) with 1% of the channels (seeded) scaled x8 as outliers
        ch = torch.randperm(d, generator=torch.Generator().manual_seed(1))[: max(1, d // 100)].to("cuda")
        for pool in (full.k_pool, full.v_pool):
            x = torch.randn(pool.shape, generator=g, device="cuda")
            x[..., ch] *= 8.0
            pool.copy_(x.to(torch.bfloat16))
        for b in range(B):
            full.set_length(b, ctx)
        return full

    if args.kernel == "draft-attn":
        full = full_cache()
        cfg = CompressionConfig(args.bits, args.keep, 4, 512)
        comp = CompressedKVCache(1, cfg, n_kv=n_kv, d_head=d, dtype="bf16", capacity=int(ctx * args.keep) + 64,
                                 batch=B, max_bits=args.bits)
        comp.sync_from(full, 0)
        kept = int(comp.meta_t[0, 0, 1])
        del full
        torch.cuda.empty_cache()
        dims = comp.dims()
        work = torch.zeros(int(_lib.load().dkv_attn_work_bytes(dims, G, 1, ctx + 64, 512, comp.cap)),
                           dtype=torch.uint8, device="cuda")
        q = torch.randn((B, n_kv * G, d), device="cuda")
        qpos = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
        out = torch.zeros((B, n_kv * G * d), dtype=torch.bfloat16, device="cuda")
        by = B * n_kv * kept * 2 * cfg.bytes_per_entry(d)
        us = timeit(lambda: _lib.call("dkv_attn_comp", comp.struct(), dims, 0, G, q.data_ptr(), qpos.data_ptr(),
                                      out.data_ptr(), _lib.BF16, work.data_ptr(), work.numel(), _lib.stream_ptr()))
        line["config"] = {"batch": B, "ctx": ctx, "kept": kept, "bits": args.bits, "keep": args.keep,
                          "n_kv": n_kv, "d_head": d, "group": G}
    elif args.kernel in ("verify-attn", "prefill-attn"):
        full = full_cache()
        prefill = args.kernel == "prefill-attn"
        T = args.T or (512 if prefill else 9)
        split = args.split or (16384 if prefill else 512)
        work = torch.zeros(int(_lib.load().dkv_attn_work_bytes(full.dims(), G, T, ctx + 64, split, 0)),
                           dtype=torch.uint8, device="cuda")
        qv = torch.randn((B * T, n_kv * G, d), device="cuda")
        p0 = torch.full((B,), ctx - T, dtype=torch.int32, device="cuda")
        outv = torch.zeros((B * T, n_kv * G * d), dtype=torch.bfloat16, device="cuda")
        by = B * n_kv * ctx * 2 * d * 2
        # causal: query t (position ctx - T + t) sees ctx - T + t + 1 keys; 4 flops a (key, dim) pair
        line["flops"] = B * n_kv * G * sum(ctx - T + t + 1 for t in range(T)) * d * 4
        us = timeit(lambda: _lib.call("dkv_attn_full", full.struct(), full.dims(), 0, G, T, qv.data_ptr(),
                                      p0.data_ptr(), outv.data_ptr(), _lib.BF16, split, work.data_ptr(), work.numel(),
                                      _lib.stream_ptr()))
        line["config"] = {"batch": B, "ctx": ctx, "T": T, "n_kv": n_kv, "d_head": d, "group": G, "split": split,
                          "pages": "allocation order" if (args.no_shuffle or prefill) else "shuffled (seed 7)"}
    elif args.kernel == "gemm-layer":
        N, NL = args.N, 8
        shapes = [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)]
        g = torch.Generator(device="cuda").manual_seed(0)
        Ws = [[_lib.pack_weight((torch.randn((M, K), generator=g, device="cuda") * 0.02).to(torch.bfloat16))
               for M, K in shapes] for _ in range(NL)]
        Xs = [torch.randn((N, K), generator=g, device="cuda").to(torch.bfloat16) for M, K in shapes]
        outs = [torch.zeros((N, M), dtype=torch.float32, device="cuda") for M, K in shapes]
        work = torch.zeros(4096, dtype=torch.uint8, device="cuda")
        epis = []
        for (M, K), o in zip(shapes, outs):
            e = _lib.EpilogueS()
            e.kind = _lib.EPI_STORE
            e.out_f32 = o.data_ptr()
            e.ld_out = M
            e.act_dtype = _lib.BF16
            epis.append(e)

        def layers():
            for l in range(NL):
                for (M, K), w, x, e in zip(shapes, Ws[l], Xs, epis):
                    _lib.call("dkv_gemm", x.data_ptr(), _lib.BF16, w.data_ptr(), _lib.BF16, M, N, K, C.byref(e),
                              work.data_ptr(), work.numel(), _lib.stream_ptr())

        layers()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            layers()
        for _ in range(3):
            graph.replay()
        ts = []
        for _ in range(iters):
            torch.cuda._sleep(100_000)
            a = torch.cuda.Event(enable_timing=True)
            b_ = torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b_.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b_) * 1e3)
        us = statistics.median(ts) / NL          # per layer
        by = sum(M * K * 2 + N * K * 2 + N * M * 4 for M, K in shapes)
        line["config"] = {"shapes": shapes, "N": N, "layers": NL, "per": "layer"}
        line["l2_note"] = "8 layers of weights (3.5 GB) per replay: inputs larger than L2"
    else:
        M, K, N = args.M, args.K, args.N
        g = torch.Generator(device="cuda").manual_seed(0)
        W = (torch.randn((M, K), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        Wt = _lib.pack_weight(W)
        del W
        X = torch.randn((N, K), generator=g, device="cuda").to(torch.bfloat16)
        out = torch.zeros((N, M), dtype=torch.float32, device="cuda")
        work = torch.zeros(int(_lib.load().dkv_gemm_work_bytes(M, N, K, _lib.BF16)), dtype=torch.uint8,
                           device="cuda")
        e = _lib.EpilogueS()
        e.kind = _lib.EPI_STORE
        e.out_f32 = out.data_ptr()
        e.ld_out = M
        e.act_dtype = _lib.BF16
        by = M * K * 2 + N * K * 2 + N * M * 4
        us = timeit(lambda: _lib.call("dkv_gemm", X.data_ptr(), _lib.BF16, Wt.data_ptr(), _lib.BF16, M, N, K,
                                      C.byref(e), work.data_ptr(), work.numel(), _lib.stream_ptr()))
        line["config"] = {"M": M, "K": K, "N": N}
    gbs = by / (us * 1e-6) / 1e9
    if "flops" in line:
        tf = line["flops"] / (us * 1e-6) / 1e12
        line.update({"achieved_tflops": round(tf, 1), "peak_tflops": round(pk["bf16_tflops"], 1),
                     "tensor_frac": round(tf / pk["bf16_tflops"], 4)})
    line.update({"us": round(us, 2), "algorithmic_bytes": int(by), "achieved_gbs": round(gbs, 1),
                 "peak_gbs": round(pk["hbm_gbs"], 1), "frac": round(gbs / pk["hbm_gbs"], 4),
                 "peak_source": pk["source"],
                 "l2": line.pop("l2_note", "flushed between launches (256 MB write)"),
                 "timing": "CUDA events on the launching stream, queued behind a device-side sleep (device time only)"})
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--rounds-per-step", type=int, default=10,
                    help="draft/verify rounds in one step (the step is the timed unit)")
    ap.add_argument("--fixed-rounds", type=int, default=100,
                    help="rounds of the always-drafting leg (8b/keep1, gamma 2)")
    ap.add_argument("--no-fixed-arm", action="store_true", help="skip the always-drafting leg")
    ap.add_argument("--prof-rounds", type=int, default=60,
                    help="rounds timed again with per-launch CUDA events (kernel roofline)")
    ap.add_argument("--config", default="c4", choices=list(CONFIGS))
    ap.add_argument("--impl", default="draftkv", choices=["draftkv", "reference"])
    ap.add_argument("--ctx", type=int, default=None)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--settle", type=int, default=60,
                    help="untimed controller-settle rounds after the warm-up (Thompson-controlled configs)")
    ap.add_argument("--split-keys", type=int, default=0,
                    help="keys per attention split (multiple of 64; default: chosen from the shape)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-calibrate", action="store_true",
                    help="keep the cost model's default fixed costs instead of measuring them on the device")
    ap.add_argument("--kernel", choices=["draft-attn", "verify-attn", "prefill-attn", "gemm", "gemm-layer"], default=None,
                    help="time one kernel alone on a synthetic case instead of the decode step")
    ap.add_argument("--bits", type=int, default=4)
    ap.add_argument("--keep", type=float, default=0.25)
    ap.add_argument("--T", type=int, default=None, help="query tokens (verify-attn 9, prefill-attn 512)")
    ap.add_argument("--M", type=int, default=28672)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--N", type=int, default=4)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--split", type=int, default=None, help="keys per split (verify-attn 512, prefill-attn 16384)")
    ap.add_argument("--no-shuffle", action="store_true", help="kernel mode: keep the page table in allocation order")
    args = ap.parse_args()
    if args.kernel:
        run_kernel(args)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
