"""The draft / verify loop on the device.

Same contract as the reference's draftkv/engine.py:44-223:

    caches hold K/V for positions 0 .. len(tokens) - 2
    the pending token tokens[-1] is never cached

Each round: the controller picks (config, gamma) on the host; gamma draft
forwards run over the compressed cache (T = 1, sampling on device), one
(gamma+1)-token verify forward runs over the full cache, acceptance
(greedy first-argmax match, or the speculative-sampling rule with the
residual resample) runs on device, the full cache is rolled back (host page
bookkeeping only) and the drafter cache is resynced from the true K/V by one
fused kernel.  Only (accepted, emitted tokens) per sequence come back to the
host, where the controller is updated.

Batching: `generate_batch` decodes several independent sequences together
(one device state, one round loop).  A round uses one (config, gamma) for the
whole batch -- the controller is asked once per round with the longest
context -- and each sequence keeps its own accepted count, which is reported
to the controller per sequence.  `generate` / `generate_baseline` are the
reference's batch-1 entry points.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .dist import ControllerExchange, replicated_select, replicated_update
from . import _lib
from .compress import CompressedKVCache
from .config import CompressionConfig, layer_cfgs
from .controller import Controller, FixedPolicy
from .paged import PagedKVCache

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


@dataclass
class RoundLog:
    cfg: CompressionConfig
    gamma: int
    accepted: int
    emitted: int
    ctx: int


@dataclass
class GenerationResult:
    tokens: list
    rounds: list = field(default_factory=list)
    draft_steps: int = 0
    verify_passes: int = 0
    cache_rebuilds: int = 0
    layers_rebuilt: int = 0

    @property
    def new_tokens(self) -> int:
        return sum(r.emitted for r in self.rounds)

    @property
    def acceptance_rate(self) -> float:
        drafted = sum(r.gamma for r in self.rounds)
        return sum(r.accepted for r in self.rounds) / drafted if drafted else float("nan")

    @property
    def tokens_per_verify(self) -> float:
        return self.new_tokens / self.verify_passes if self.verify_passes else float("nan")


class _Batch:
    """Device state of one generate call: caches, token ring, buffers."""

    def __init__(self, eng: "DraftKVEngine", prompts: list, max_new: int, gamma_max: int,
                 temperature: float, page_size: int = 16) -> None:
        m = eng.model
        self.m = m
        self.B = B = len(prompts)
        self.G = gamma_max
        self.VS = gamma_max + 2                     # token ring stride per sequence
        self.max_ctx = max(len(p) for p in prompts) + max_new + gamma_max + 2
        m.ensure_positions(self.max_ctx)
        pages = -(-self.max_ctx // page_size)
        if eng.full_cache_factory is not None:
            # the reference's factory takes no arguments and returns one cache
            self.full = eng.full_cache_factory()
            if hasattr(self.full, "materialize"):
                self.full.materialize(m.n_kv_heads, m.d_head, m.dtype)
                self.full.grow(self.max_ctx)
            if getattr(self.full, "batch", 1) != B:
                raise ValueError("full_cache_factory must return a cache with one slot per sequence")
            if self.full.capacity_tokens < self.max_ctx:
                raise ValueError(f"full cache holds {self.full.capacity_tokens} positions < {self.max_ctx}")
        else:
            self.full = PagedKVCache(m.n_layers, m.n_kv_heads, m.d_head, page_size, pages * m.n_layers * B, m.dtype,
                                     batch=B, max_blocks_per_seq=pages)
        dev = m.device
        self.vtok = torch.zeros((B, self.VS), dtype=torch.int32, device=dev)
        self.base_pos = torch.zeros((B,), dtype=torch.int32, device=dev)
        self.accepted = torch.zeros((B,), dtype=torch.int32, device=dev)
        self.next = torch.zeros((B,), dtype=torch.int32, device=dev)
        self.rs = torch.zeros((3, B), dtype=torch.int32, device=dev)
        self.active = torch.ones((B,), dtype=torch.int32, device=dev)
        self.counters = torch.zeros((gamma_max + 2,), dtype=torch.int64, device=dev)
        self.pos_draft = torch.zeros((max(gamma_max, 1), B), dtype=torch.int32, device=dev)
        self.ctr_host = torch.zeros((gamma_max + 2,), dtype=torch.int64, pin_memory=True)
        V = m.vocab_size
        self.draft_logits = torch.zeros((max(gamma_max, 1), B, V), dtype=torch.float32, device=dev)
        self.verify_logits = torch.zeros((B, gamma_max + 1, V), dtype=torch.float32, device=dev)
        self.accept_work = torch.zeros(int(_lib.load().dkv_sample_work_bytes(B, V)), dtype=torch.uint8, device=dev)
        cap = 0
        self.comp: CompressedKVCache | None = None
        self.work = None
        self._cap = cap
        self.host_acc = torch.zeros((B,), dtype=torch.int32, pin_memory=True)
        self.host_tok = torch.zeros((B, self.VS), dtype=torch.int32, pin_memory=True)

    def workspace(self):
        cap = self.comp.cap if self.comp is not None else 0
        if self.work is None or self._cap != cap:
            self.work = self.m.work(self.B, self.G + 1, self.full.capacity_tokens, cap)
            self._cap = cap
        return self.work


class DraftKVEngine:
    """Self-speculative decoding with the target model drafting from a
    compressed copy of its own KV cache (engine.py:76-223).  Output equals
    full-KV decoding exactly under greedy decoding and in distribution under
    sampling."""

    def __init__(self, model, controller: Controller | None = None, seed: int = 0,
                 full_cache_factory=None, gamma_max: int | None = None) -> None:
        self.model = model
        self.controller = controller or FixedPolicy(CompressionConfig(4, 0.5), 4)
        self.seed = int(seed)
        # keep the full cache in pinned host memory after the prefill (the
        # drafter cache stays in HBM); verify streams it over the host link
        self.offload_full = False
        # prompt tokens per sequence in one prefill forward (prompts of 1024
        # tokens or more; shorter ones take 64): at least prefill_chunk, and
        # prefill_tokens over the batch, so that a forward's projections see
        # ~2048 tokens (256-token GEMM tiles; 512 tokens a launch ran the
        # Llama-3-8B shape's projections at 318 TF/s on B200)
        self.prefill_chunk = 512
        self.prefill_tokens = 2048

        self.full_cache_factory = full_cache_factory
        self.gamma_max = gamma_max
        self._round = 0
        # CUDA events around the phases of each round and around rebuilds
        # (None: off).  calibrate.py turns this on to measure the device's
        # own draft / verify / resync / rebuild costs.
        self.phase_events: list | None = None
        self.rebuild_events: list | None = None

    # ---------------------------------------------------------------- util
    def _gamma_max(self) -> int:
        if self.gamma_max is not None:
            return self.gamma_max
        g = getattr(self.controller, "gamma_max", None)
        if g is None and isinstance(self.controller, FixedPolicy):
            g = self.controller.gamma
        return int(g or 8)

    def _set_counters(self, st: _Batch) -> None:
        self._round += 1
        base = self._round * 64
        for i in range(st.G + 2):
            st.ctr_host[i] = base + i
        st.counters.copy_(st.ctr_host, non_blocking=True)

    def _prefill(self, st: _Batch, prompts: list) -> None:
        """Writes K/V of prompt[:-1] for every sequence (engine.py:133-134),
        in chunks, through the full-cache forward."""
        m, B = self.model, st.B
        lens = [len(p) - 1 for p in prompts]
        L = max(lens) if lens else 0
        CH = max(self.prefill_chunk, self.prefill_tokens // max(B, 1)) if L >= 1024 else 64
        tok = torch.zeros((B, max(L, 1)), dtype=torch.int32)
        for b, p in enumerate(prompts):
            if lens[b] > 0:
                tok[b, :lens[b]] = torch.tensor(p[:-1], dtype=torch.int32)
        tok = tok.to(m.device)
        work = m.work(B, CH, st.full.capacity_tokens, 0)
        for b in range(B):
            st.full.ensure(b, lens[b] + st.G + 2)
        for c0 in range(0, L, CH):
            c1 = min(L, c0 + CH)
            # sequences shorter than the chunk start re-write their own last
            # rows harmlessly; rows past a sequence's prompt are never read
            pos0 = torch.full((B,), c0, dtype=torch.int32, device=m.device)
            tok_c = tok[:, c0:c1].contiguous()
            # no logits: the reference discards the prompt's (engine.py:133-134)
            m.forward_raw(st.full, None, tok_c.data_ptr(), c1 - c0, pos0, B, c1 - c0, None, work, CH,
                          st.full.capacity_tokens, graph=False)
        for b in range(B):
            st.full.set_length(b, lens[b])

    def _start(self, prompts: list, max_new: int, temperature: float) -> _Batch:
        for p in prompts:
            if len(p) < 1:
                raise ValueError("prompt must hold at least one token")
        st = _Batch(self, prompts, max_new, self._gamma_max(), temperature)
        if any(len(p) != len(prompts[0]) for p in prompts):
            raise ValueError("generate_batch needs prompts of one length")
        self._prefill(st, prompts)
        if self.offload_full and hasattr(st.full, "offload_to_host"):
            st.full.offload_to_host()
        pend = torch.tensor([p[-1] for p in prompts], dtype=torch.int32)
        st.vtok[:, 0] = pend.to(st.vtok.device)
        st.base_pos.fill_(len(prompts[0]) - 1)
        return st

    # ---------------------------------------------------------- baseline
    def generate_baseline(self, prompt: list, max_new_tokens: int, temperature: float = 0.0) -> list:
        """Plain full-KV autoregressive decoding (engine.py:109-120)."""
        return self.generate_baseline_batch([prompt], max_new_tokens, temperature)[0]

    def generate_baseline_batch(self, prompts: list, max_new_tokens: int, temperature: float = 0.0) -> list:
        st = self._start([list(p) for p in prompts], max_new_tokens, temperature)
        toks = [list(p) for p in prompts]
        for _ in range(max_new_tokens):
            self._baseline_step(st, temperature)
            torch.cuda.current_stream().synchronize()
            nxt = st.next.cpu().tolist()
            for b in range(st.B):
                toks[b].append(int(nxt[b]))
        return toks

    def _baseline_step(self, st: _Batch, temperature: float) -> None:
        """One T = 1 forward over the full cache plus a draw; the same kernels
        as the verify pass, so each token equals the verify pass's row."""
        m = self.model
        n = [st.full.counts[b][0] for b in range(st.B)]
        for b in range(st.B):
            st.full.ensure(b, n[b] + 1)
        self._set_counters(st)
        work = st.workspace()

        def body():
            m.forward_raw(st.full, None, st.vtok.data_ptr(), st.VS, st.base_pos, st.B, 1, st.verify_logits, work,
                          st.G + 1, st.full.capacity_tokens)
            _lib.call("dkv_accept", st.verify_logits.data_ptr(), None, st.B, 0, m.vocab_size, float(temperature),
                      self.seed, st.counters[st.G + 1:].data_ptr(), st.vtok.data_ptr(), st.VS,
                      st.base_pos.data_ptr(), st.accepted.data_ptr(), st.next.data_ptr(), st.rs[0].data_ptr(),
                      st.rs[1].data_ptr(), st.rs[2].data_ptr(), st.active.data_ptr(), st.accept_work.data_ptr(),
                      st.accept_work.numel(), _lib.stream_ptr())

        body()
        for b in range(st.B):
            st.full.set_length(b, n[b] + 1)

    # ---------------------------------------------------------- draftkv
    def generate(self, prompt: list, max_new_tokens: int, temperature: float = 0.0,
                 context_key: str | None = None) -> GenerationResult:
        """engine.py:123-223 for one prompt."""
        return self.generate_batch([prompt], max_new_tokens, temperature, context_key)[0]

    def generate_batch(self, prompts: list, max_new_tokens: int, temperature: float = 0.0,
                       context_key: str | None = None, exchange=None) -> list:
        """Decodes several same-length prompts together; one result each."""
        sess = self.session(prompts, max_new_tokens, temperature, context_key, exchange)
        while not sess.done:
            sess.round()
        sess.finish()
        return sess.results()

    def session(self, prompts: list, max_new_tokens: int, temperature: float = 0.0,
                context_key: str | None = None, exchange=None) -> "Session":
        """Prefills `prompts` and returns a Session whose round() runs one
        draft / verify round.  `exchange` (see draftkv.dist), when given,
        replicates the controller's inputs over processes: a
        ControllerExchange (batched, asynchronous) or a per-round exchange
        function; the controller selects on the largest context over all
        processes and is updated with every process's (accepted, context,
        gamma), so replicated controllers stay identical.  Every process must
        call round() the same number of times, then finish()."""
        return Session(self, [list(p) for p in prompts], max_new_tokens, temperature, context_key, exchange)

    # -------------------------------------------------------- device round
    def _new_comp(self, st: _Batch, cfg) -> CompressedKVCache:
        m = self.model
        arms = getattr(self.controller, "arms", None) or [cfg]
        cfgs = [c for a in arms for c in layer_cfgs(a, m.n_layers)] + layer_cfgs(cfg, m.n_layers)
        max_bits = max(c.bits for c in cfgs)
        cap = self._comp_slots(st, cfgs)
        comp = CompressedKVCache(m.n_layers, layer_cfgs(cfg, m.n_layers), batch=st.B, capacity=cap,
                                 max_bits=max_bits)
        comp.materialize(m.n_kv_heads, m.d_head, m.dtype)
        return comp

    @staticmethod
    def _comp_slots(st: _Batch, cfgs) -> int:
        """Slots a drafter cache needs for per-layer configs `cfgs`."""
        cap = 0
        for c in cfgs:
            kept = max(int(round(c.keep_frac * st.max_ctx)), c.sink + c.recent)
            cap = max(cap, min(kept, st.max_ctx))
        return cap + st.G + 4

    def _comp_too_small(self, st: _Batch, cfgs) -> bool:
        comp = st.comp
        return max(c.bits for c in cfgs) > comp.max_bits or self._comp_slots(st, cfgs) > comp.cap

    def _rebuild(self, st: _Batch, layers: list, ctx_t, advance: bool) -> None:
        if not layers:
            return
        import ctypes as C
        if advance and 0 in layers and len(layers) == self.model.n_layers:
            st.comp.seen_t.zero_()
        arr = (C.c_int32 * len(layers))(*layers)
        ev = self._event() if self.rebuild_events is not None else None
        _lib.call("dkv_comp_rebuild", st.comp.struct(), st.full.struct(), st.comp.dims(), arr, len(layers),
                  ctx_t.data_ptr(), 1 if advance else 0, _lib.stream_ptr())
        if ev is not None:
            self.rebuild_events.append((len(layers), ev, self._event()))

    @staticmethod
    def _event():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def _resync(self, st: _Batch) -> None:
        """comp.sync_from(full, n-1) with (pos0, rows, trunc) computed on device
        by the acceptance kernel."""
        m = self.model
        _lib.call("dkv_comp_append", st.comp.struct(), st.full.struct(), st.comp.dims(), 0, m.n_layers, None,
                  m.dtype, st.G + 1, st.rs[0].data_ptr(), st.rs[1].data_ptr(), st.rs[2].data_ptr(), 1,
                  _lib.stream_ptr())

    def _round_device(self, st: _Batch, gamma: int, temperature: float) -> None:
        m = self.model
        work = st.workspace()
        V = m.vocab_size
        ev = [self._event()] if self.phase_events is not None else None
        for i in range(gamma):
            pos_i = st.pos_draft[i]
            torch.add(st.base_pos, i, out=pos_i)
            m.forward_raw(None, st.comp, st.vtok.data_ptr() + 4 * i, st.VS, pos_i, st.B, 1, st.draft_logits[i], work,
                          st.G + 1, st.full.capacity_tokens)
            _lib.call("dkv_sample", st.draft_logits[i].data_ptr(), st.B, V, float(temperature), self.seed,
                      st.counters[i:].data_ptr(), st.vtok.data_ptr() + 4 * (i + 1), st.VS, None, 0,
                      _lib.stream_ptr())
        if ev is not None:
            ev.append(self._event())
        m.forward_raw(st.full, None, st.vtok.data_ptr(), st.VS, st.base_pos, st.B, gamma + 1, st.verify_logits,
                      work, st.G + 1, st.full.capacity_tokens)
        _lib.call("dkv_accept", st.verify_logits.data_ptr(), st.draft_logits.data_ptr(), st.B, gamma, V,
                  float(temperature), self.seed, st.counters[st.G + 1:].data_ptr(), st.vtok.data_ptr(), st.VS,
                  st.base_pos.data_ptr(), st.accepted.data_ptr(), st.next.data_ptr(), st.rs[0].data_ptr(),
                  st.rs[1].data_ptr(), st.rs[2].data_ptr(), st.active.data_ptr(), st.accept_work.data_ptr(),
                  st.accept_work.numel(), _lib.stream_ptr())
        if ev is not None:
            ev.append(self._event())
        self._resync(st)
        if ev is not None:
            ev.append(self._event())
            self.phase_events.append((gamma, ev))

    def _collect(self, st: _Batch, gamma: int) -> list:
        """(accepted, emitted tokens) per sequence -- the only device->host read."""
        st.host_acc.copy_(st.accepted, non_blocking=True)
        st.host_tok.copy_(st.vtok, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        acc = st.host_acc.numpy()
        tok = st.host_tok.numpy()
        out = []
        for b in range(st.B):
            k = int(acc[b])
            # vtok[b] = [pending, drafts..., ] with the emitted stream at 1..k+1
            out.append((k, [int(t) for t in tok[b, 1:1 + k + 1]]))
        return out


class Session:
    """One batched generation in progress (see DraftKVEngine.session)."""

    def __init__(self, eng: DraftKVEngine, prompts: list, max_new: int, temperature: float, key, exchange) -> None:
        self.eng = eng
        self.m = eng.model
        self.T = float(temperature)
        self.key = key
        self.exchange = exchange
        self.max_new = max_new
        self.st = eng._start(prompts, max_new, temperature)
        self.B = self.st.B
        self.toks = [list(p) for p in prompts]
        self.res = [GenerationResult(tokens=self.toks[b]) for b in range(self.B)]
        self.plen = len(prompts[0])
        self.comp_cfg = None
        self.last = None        # (cfg, gamma, [(k, emitted)]) of the latest round
        self.batched = isinstance(exchange, ControllerExchange)
        if self.batched:
            exchange.start(max(len(p) for p in prompts))

    def _select(self, n: list):
        if self.batched:
            return self.exchange.select(self.eng.controller, self.key)
        # every process selects on the same (largest) context
        return replicated_select(self.eng.controller, max(n), self.key, self.exchange)

    def _update(self, cfg, records: list) -> None:
        """records: (accepted, context, gamma, next context) per active
        sequence of this process (accepted < 0: context only)."""
        if self.batched:
            self.exchange.update(records)
            return
        replicated_update(self.eng.controller, cfg, [(k, c, g) for k, c, g, _n in records if k >= 0], self.key,
                          self.exchange)

    def finish(self) -> None:
        """Applies every outstanding exchange batch (every process calls it
        once, after its last round)."""
        if self.batched:
            self.exchange.finish(self.eng.controller, self.key)

    @property
    def done(self) -> bool:
        return all(len(t) - self.plen >= self.max_new for t in self.toks)

    def results(self) -> list:
        for b in range(self.B):
            self.res[b].tokens = self.toks[b]
        return self.res

    def round(self) -> list:
        """One round for every active sequence; returns [(accepted, emitted)]."""
        eng, st, m, B = self.eng, self.st, self.m, self.B
        left = [self.max_new - (len(self.toks[b]) - self.plen) for b in range(B)]
        active = [lft > 0 for lft in left]
        n = [len(self.toks[b]) for b in range(B)]
        # every process selects on the same context: replicated controllers
        # stay identical
        cfg, gamma = self._select(n)
        if not any(active):
            self._update(cfg, [])
            return []
        gamma = min(gamma, max(min(l for l, a in zip(left, active) if a) - 1, 0), st.G)
        st.active.copy_(torch.tensor([1 if a else 0 for a in active], dtype=torch.int32), non_blocking=True)
        eng._set_counters(st)
        if gamma <= 0:
            eng._baseline_step(st, self.T)
            if st.comp is not None:
                eng._resync(st)
            out = eng._collect(st, 0)
            for b in range(B):
                if active[b]:
                    self.toks[b].append(out[b][1][0])
                    self.res[b].verify_passes += 1
                    self.res[b].rounds.append(RoundLog(cfg, 0, 0, 1, n[b]))
            # every process takes part in every round's exchange
            self._update(cfg, [(-1, n[b], 0, n[b] + 1) for b in range(B) if active[b]])
            self.last = (cfg, 0, out)
            return out
        # drafter cache: create, or rebuild only the layers whose config changed
        if st.comp is None:
            st.comp = eng._new_comp(st, cfg)
            ctx_t = torch.tensor([n[b] - 1 for b in range(B)], dtype=torch.int32, device=m.device)
            eng._rebuild(st, list(range(m.n_layers)), ctx_t, advance=True)
            self.comp_cfg = cfg
            for r in self.res:
                r.cache_rebuilds += 1
        elif self.comp_cfg != cfg:
            old = layer_cfgs(self.comp_cfg, m.n_layers)
            new = layer_cfgs(cfg, m.n_layers)
            if eng._comp_too_small(st, new):
                # wider codes or a larger budget than the cache was sized for
                # (a policy switched to an arm outside the controller's set):
                # a new cache, every layer rebuilt
                st.comp = eng._new_comp(st, cfg)
                changed = list(range(m.n_layers))
            else:
                changed = [L for L in range(m.n_layers) if old[L] != new[L]]
                st.comp.set_cfgs(new)
            ctx_t = torch.tensor([n[b] - 1 for b in range(B)], dtype=torch.int32, device=m.device)
            eng._rebuild(st, changed, ctx_t, advance=0 in changed)
            self.comp_cfg = cfg
            for r in self.res:
                r.cache_rebuilds += 1
                r.layers_rebuilt += len(changed)
        for b in range(B):
            st.full.ensure(b, n[b] + gamma)
        eng._round_device(st, gamma, self.T)
        out = eng._collect(st, gamma)            # the one device -> host read
        stats = []
        for b in range(B):
            k, emitted = out[b]
            if not active[b]:
                st.full.set_length(b, n[b] - 1)
                continue
            self.toks[b].extend(emitted)
            st.full.set_length(b, n[b] - 1 + gamma + 1)
            st.full.truncate_seq(b, n[b] + k)        # rollback (engine.py:216)
            stats.append((k, n[b], gamma, n[b] + len(emitted)))
            self.res[b].draft_steps += gamma
            self.res[b].verify_passes += 1
            self.res[b].rounds.append(RoundLog(cfg, gamma, k, len(emitted), n[b]))
        self._update(cfg, stats)
        self.last = (cfg, gamma, out)
        return out
