"""Per-layer damage model and the exact byte-budget allocator.

The parts of the reference's draftkv/layers.py that the online layer
allocator (adaptive.py) runs on: the damage table `SensitivityProfile`
(layers.py:82-127, the fields and the separable objective; the offline
profiling runs that fill it from model passes are not part of the decode
step) and `allocate` (layers.py:301-368), the exact multiple-choice knapsack
that picks one configuration per layer to minimise the summed damage under a
byte budget.  Host policy: no device work.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .config import CompressionConfig, LayerPlan


@dataclass
class SensitivityProfile:
    """Acceptance with one layer degraded at a time (layers.py:82-127).

    `alpha[(layer, cfg)]` is the acceptance measured (or predicted) with only
    `layer` at `cfg`; missing cells read as `alpha_ref`.  `p` is the
    composition exponent of the objective (1 = log-additive damages)."""

    reference: CompressionConfig
    alpha_ref: float
    candidates: tuple
    alpha: dict = field(default_factory=dict)
    trials: dict = field(default_factory=dict)
    spread: dict = field(default_factory=dict)
    p: float = 1.0
    n_prompts: int = 1

    def damage(self, layer: int, cfg: CompressionConfig) -> float:
        """log alpha_ref - log alpha(layer at cfg), never negative."""
        a = self.alpha.get((layer, cfg), self.alpha_ref)
        return max(0.0, float(np.log(max(self.alpha_ref, 1e-6)) - np.log(max(a, 1e-6))))

    def objective(self, layer: int, cfg: CompressionConfig) -> float:
        return self.damage(layer, cfg) ** self.p

    def composed_damage(self, plan: LayerPlan) -> float:
        tot = sum(self.objective(L, c) for L, c in enumerate(plan))
        return float(tot ** (1.0 / self.p)) if tot > 0 else 0.0

    def predicted_alpha(self, plan: LayerPlan) -> float:
        return float(np.clip(self.alpha_ref * np.exp(-self.composed_damage(plan)), 0.0, 1.0))


def _ranked_costs(prof: SensitivityProfile, ctx: int, n_kv_heads: int, d_head: int):
    """Candidates cheapest first (stable) with the bytes one layer of each costs."""
    def one(c):
        return LayerPlan((c,)).per_layer_bytes(ctx, n_kv_heads, d_head)

    ranked = sorted(prof.candidates, key=one)
    return ranked, [one(c) for c in ranked]


def allocate(prof: SensitivityProfile, budget_bytes: float, ctx: int, n_kv_heads: int, d_head: int,
             n_layers: int, max_states: int = 20000) -> LayerPlan:
    """Exact multiple-choice knapsack (layers.py:301-368).

    Layer by layer, carry the Pareto frontier of (bytes, damage) partial plans
    in exact byte counts (no bucketing), keeping a state only if it damages
    strictly less than every cheaper one, and reserving the cheapest
    configuration's bytes for the layers still to come.  The plan of least
    total damage on the final frontier (first on ties) is returned; the
    all-cheapest plan when even that does not fit.  `max_states` bounds the
    frontier by keeping its lowest-damage states."""
    ranked, costs = _ranked_costs(prof, ctx, n_kv_heads, d_head)
    cheapest = LayerPlan(tuple(ranked[0] for _ in range(n_layers)))
    if costs[0] * n_layers > budget_bytes + 1e-9:
        return cheapest
    frontier = [(0.0, 0.0)]
    parents: list = []
    for L in range(n_layers):
        later = costs[0] * (n_layers - L - 1)
        cand = []
        for pi, (b0, d0) in enumerate(frontier):
            for j, cfg in enumerate(ranked):
                b = b0 + costs[j]
                if b + later > budget_bytes + 1e-9:
                    continue
                cand.append((b, d0 + prof.objective(L, cfg), j, pi))
        if not cand:
            return cheapest
        cand.sort(key=lambda s: (s[0], s[1]))
        keep, lowest = [], float("inf")
        for s in cand:
            if s[1] < lowest - 1e-12:
                keep.append(s)
                lowest = s[1]
        if len(keep) > max_states:
            keep = sorted(keep, key=lambda s: s[1])[:max_states]
            keep.sort(key=lambda s: (s[0], s[1]))
        frontier = [(b, d) for b, d, _, _ in keep]
        parents.append([(j, pi) for _, _, j, pi in keep])
    at = min(range(len(frontier)), key=lambda i: frontier[i][1])
    picks = []
    for L in range(n_layers - 1, -1, -1):
        j, at = parents[L][at]
        picks.append(j)
    return LayerPlan(tuple(ranked[j] for j in reversed(picks)))
