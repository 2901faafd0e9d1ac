"""Online per-layer budget allocation (reference draftkv/adaptive.py:68-335).

`AdaptiveLayerController` is a controller (select / update) whose `select`
returns a `LayerPlan`: one compression configuration per layer, chosen to
maximise acceptance under a byte budget for the drafter cache.  The engine
takes a plan wherever it takes a configuration; on a plan change it rebuilds
only the layers whose configuration changed (the device rebuild kernel takes
a list of layers), which is what makes online probing affordable.

How it learns (same rule and the same order of random draws as the
reference, so a seeded run makes the same decisions):
  * most rounds run the current plan and update a Beta posterior of the
    plan's per-token acceptance;
  * with probability `effective_probe_prob(ctx)` a round runs a *swap probe*:
    one notch of budget moved from layer `down` to layer `up` (only pairs that
    fit the budget are enumerated; the least-probed `up` is preferred, ties
    broken by one uniform draw).  Its acceptance, relative to the base rate in
    log space, is credited to `up` and debited from `down` with rate `lr`
    (paired comparison, so layers pinned at either end keep being measured);
  * every `resolve_every` decisions the knapsack (layers.allocate) is re-solved
    from the shifted values, with damage extrapolated linearly in notches,
    and any unspent budget buys upgrades for the layers that hurt most;
  * a run of `stall_limit` gamma-0 decisions resets the plan to the most
    generous one the budget allows (a gamma-0 round measures nothing);
  * the probe rate is capped so that the rebuilds a probe causes (two
    layers, there and back: CostModel.rebuild_cost) cost at most
    `max_probe_overhead` of a round.
Everything is keyed by the caller's context key.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from .config import CompressionConfig, LayerPlan
from .controller import _Beta
from .layers import SensitivityProfile, allocate
from .throughput import CostModel, best_gamma


@dataclass
class _LayerStats:
    """Base acceptance posterior and the paired-comparison value per layer."""

    base: _Beta
    value: dict = field(default_factory=dict)
    probe_n: dict = field(default_factory=dict)


class AdaptiveLayerController:
    """Controller protocol over per-layer plans (adaptive.py:68-335)."""

    def __init__(self, cost: CostModel, n_layers: int, budget_bytes: float,
                 candidates: Sequence[CompressionConfig] | None = None, ctx_hint: int = 4096,
                 gamma_max: int = 8, probe_prob: float = 0.15, max_probe_overhead: float = 0.05,
                 resolve_every: int = 64, decay: float = 0.995, lr: float = 0.08, min_speedup: float = 1.05,
                 stall_limit: int = 12, seed: int = 0, prior: tuple = (2.0, 1.0)) -> None:
        self.cost = cost
        self.n_layers = n_layers
        self.budget_bytes = budget_bytes
        self.candidates = tuple(candidates or [CompressionConfig(4, 0.25), CompressionConfig(4, 0.5),
                                               CompressionConfig(4, 1.0)])
        self.ranked = tuple(sorted(self.candidates, key=lambda c: self._bytes_of(c, ctx_hint)))
        self.ctx_hint = ctx_hint
        self.gamma_max = gamma_max
        self.probe_prob = probe_prob
        self.max_probe_overhead = max_probe_overhead
        self.resolve_every = max(1, resolve_every)
        self.decay = decay
        self.lr = lr
        self.min_speedup = min_speedup
        self.stall_limit = max(1, stall_limit)
        self.prior = prior
        self.rng = np.random.default_rng(seed)
        self.stats: dict = {}
        self.plans: dict = {}
        self._stall: dict = {}
        self._last = None
        self.n_decisions = 0
        self.n_probes = 0
        self.n_resolves = 0
        self.n_stall_recoveries = 0

    @property
    def arms(self) -> tuple:
        """Every configuration a plan can hold (the engine sizes the drafter
        cache for the widest and longest of them)."""
        return self.ranked

    # ------------------------------------------------------------ helpers
    def _bytes_of(self, c: CompressionConfig, ctx: int) -> float:
        return LayerPlan((c,)).per_layer_bytes(ctx, self.cost.n_kv_heads, self.cost.d_head)

    def _plan_bytes(self, plan: LayerPlan) -> float:
        return plan.per_layer_bytes(self.ctx_hint, self.cost.n_kv_heads, self.cost.d_head)

    def _stats(self, key) -> _LayerStats:
        st = self.stats.get(key)
        if st is None:
            st = self.stats[key] = _LayerStats(base=_Beta(*self.prior))
        return st

    def _plan(self, key) -> LayerPlan:
        """The key's current plan; initially the most generous uniform plan
        the budget affords (the cheapest when none does)."""
        plan = self.plans.get(key)
        if plan is None:
            fits = [c for c in self.ranked
                    if self._plan_bytes(LayerPlan.uniform(c, self.n_layers)) <= self.budget_bytes]
            plan = self.plans[key] = LayerPlan.uniform(fits[-1] if fits else self.ranked[0], self.n_layers)
        return plan

    def _notch(self, i: int) -> float:
        return self._bytes_of(self.ranked[i], self.ctx_hint)

    def _swap_probe(self, base: LayerPlan, key):
        """(probe plan, up, down) moving one notch from `down` to `up` within
        the budget, or None when no pair fits."""
        idx = [self.ranked.index(c) for c in base.cfgs]
        room = self.budget_bytes - self._plan_bytes(base)
        seen = self._stats(key).probe_n
        pairs = []
        for up in range(self.n_layers):
            if idx[up] + 1 >= len(self.ranked):
                continue
            gain = self._notch(idx[up] + 1) - self._notch(idx[up])
            for down in range(self.n_layers):
                if down == up or idx[down] == 0:
                    continue
                give = self._notch(idx[down]) - self._notch(idx[down] - 1)
                if gain - give <= room + 1e-6:
                    pairs.append((seen.get(up, 0), up, down))
        if not pairs:
            return None
        least = min(p[0] for p in pairs)
        pool = [p for p in pairs if p[0] == least]
        _, up, down = pool[int(self.rng.integers(len(pool)))]
        cfgs = list(base.cfgs)
        cfgs[up] = self.ranked[idx[up] + 1]
        cfgs[down] = self.ranked[idx[down] - 1]
        return LayerPlan(tuple(cfgs)), up, down

    def effective_probe_prob(self, ctx: int) -> float:
        """min(probe_prob, the rate at which a probe's two rebuilds -- there
        and back -- cost at most max_probe_overhead of a verify round)."""
        rebuild = self.cost.rebuild_cost(ctx, layers_changed=2)
        if rebuild <= 0:
            return self.probe_prob
        per_round = self.cost.t_verify(ctx, self.gamma_max)
        return float(min(self.probe_prob, max(0.0, self.max_probe_overhead * per_round / (2.0 * rebuild))))

    # ---------------------------------------------------------------- api
    def select(self, ctx: int, key=None):
        self.n_decisions += 1
        if self.n_decisions % self.resolve_every == 0:
            self.resolve(key)
        base = self._plan(key)
        st = self._stats(key)
        plan, probed = base, None
        if self.rng.random() < self.effective_probe_prob(ctx):
            got = self._swap_probe(base, key)
            if got is not None:
                plan, up, down = got
                probed = (up, down)
                self.n_probes += 1
        self._last = (key, probed)
        g, t = best_gamma(self.cost, plan, st.base.mean, ctx, self.gamma_max)
        if g > 0 and t < self.min_speedup / self.cost.t_baseline(ctx):
            g = 0
        if g == 0:
            # a gamma-0 round runs on the full cache and says nothing about
            # the plan: a run of them counts as evidence against the plan
            self._stall[key] = self._stall.get(key, 0) + 1
            if self._stall[key] >= self.stall_limit:
                self._recover(key)
                plan = self.plans[key]
                st.base = _Beta(*self.prior)
                g, t = best_gamma(self.cost, plan, st.base.mean, ctx, self.gamma_max)
                self._last = (key, None)
        else:
            self._stall[key] = 0
        return plan, g

    def update(self, cfg, gamma: int, accepted: int, ctx: int, key=None) -> None:
        if gamma <= 0 or self._last is None:
            return
        k, probed = self._last
        st = self._stats(k)
        if probed is None:
            st.base.observe(accepted, gamma, self.decay)
            return
        up, down = probed
        delta = float(np.log(max(accepted / gamma, 1e-3)) - np.log(max(st.base.mean, 1e-3)))
        st.value[up] = (1 - self.lr) * st.value.get(up, 0.0) + self.lr * delta
        st.value[down] = (1 - self.lr) * st.value.get(down, 0.0) - self.lr * delta
        st.probe_n[up] = st.probe_n.get(up, 0) + 1
        st.probe_n[down] = st.probe_n.get(down, 0) + 1

    # ----------------------------------------------------------- planning
    def _spend_surplus(self, plan: LayerPlan, key) -> LayerPlan:
        """Upgrades, one notch at a time, the layer of largest damage (then
        the cheapest upgrade) while the budget allows."""
        dmg = self.damages(key)
        cfgs = list(plan.cfgs)
        spent = self._plan_bytes(LayerPlan(tuple(cfgs)))
        while True:
            best = None
            for L in range(self.n_layers):
                i = self.ranked.index(cfgs[L])
                if i + 1 >= len(self.ranked):
                    continue
                extra = self._bytes_of(self.ranked[i + 1], self.ctx_hint) - self._bytes_of(cfgs[L], self.ctx_hint)
                if spent + extra > self.budget_bytes:
                    continue
                score = (dmg[L], -extra)
                if best is None or score > best[0]:
                    best = (score, L, extra)
            if best is None:
                return LayerPlan(tuple(cfgs))
            _, L, extra = best
            cfgs[L] = self.ranked[self.ranked.index(cfgs[L]) + 1]
            spent += extra

    def _recover(self, key) -> None:
        self.plans[key] = self._spend_surplus(LayerPlan.uniform(self.ranked[0], self.n_layers), key)
        self._stall[key] = 0
        self.n_stall_recoveries += 1

    def damages(self, key=None) -> list:
        """Per-notch value of each layer, shifted so the least valuable is 0."""
        st = self._stats(key)
        vals = [st.value.get(L, 0.0) for L in range(self.n_layers)]
        lo = min(vals)
        return [v - lo for v in vals]

    def resolve(self, key=None) -> LayerPlan:
        """Re-solves the knapsack from the current values (damage of a deeper
        cut extrapolated linearly in notches) and spends the surplus."""
        st = self._stats(key)
        dmg = self.damages(key)
        prof = SensitivityProfile(self.ranked[-1], max(st.base.mean, 1e-4), self.ranked)
        for L in range(self.n_layers):
            for i, c in enumerate(self.ranked):
                notches = len(self.ranked) - 1 - i
                prof.alpha[(L, c)] = float(np.exp(np.log(prof.alpha_ref) - dmg[L] * notches))
        plan = allocate(prof, self.budget_bytes, self.ctx_hint, self.cost.n_kv_heads, self.cost.d_head,
                        self.n_layers)
        plan = self._spend_surplus(plan, key)
        self.plans[key] = plan
        self.n_resolves += 1
        return plan
