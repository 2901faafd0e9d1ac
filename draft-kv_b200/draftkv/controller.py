"""Online choice of (compression config, draft length) -- host policy.

The same controllers as the reference's draftkv/controller.py:29-335, with
the same decision rule and the same order of random draws (so a seeded run
makes the same choices): Thompson sampling over configs with gamma solved
from the sampled acceptance rate, a depth-indexed variant, a flat
(config, gamma) bandit, an oracle and a fixed policy.

The device engine feeds these only (accepted, gamma) per sequence per round;
the policy itself stays on the host, where it costs microseconds per round.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol, Sequence

import numpy as np

from .config import CompressionConfig, default_arms
from .throughput import CostModel, best_gamma, best_gamma_profile


class Controller(Protocol):
    def select(self, ctx: int, key: str | None = None) -> tuple[CompressionConfig, int]: ...

    def update(self, cfg: CompressionConfig, gamma: int, accepted: int, ctx: int,
               key: str | None = None) -> None: ...


@dataclass
class FixedPolicy:
    """One config and one gamma for every round (controller.py:36-47)."""

    cfg: CompressionConfig
    gamma: int

    def select(self, ctx: int, key: str | None = None):
        return self.cfg, self.gamma

    def update(self, cfg, gamma, accepted, ctx, key=None) -> None:
        return None


class _Beta:
    """Beta posterior on per-token acceptance; truncated-geometric update with
    decay toward the uniform prior (controller.py:50-65)."""

    __slots__ = ("a", "b")

    def __init__(self, a: float = 1.0, b: float = 1.0) -> None:
        self.a, self.b = a, b

    def observe(self, accepted: int, gamma: int, decay: float) -> None:
        self.a = 1.0 + (self.a - 1.0) * decay + accepted
        self.b = 1.0 + (self.b - 1.0) * decay + (1.0 if accepted < gamma else 0.0)

    @property
    def mean(self) -> float:
        return self.a / (self.a + self.b)

    def sample(self, rng: np.random.Generator) -> float:
        return float(rng.beta(self.a, self.b))


class ThompsonController:
    """Thompson sampling over configs; gamma = argmax of the cost model at the
    sampled alpha; challengers pay an amortized rebuild penalty; drafting is
    declined when the predicted win is under `min_speedup` (controller.py:68-170)."""

    def __init__(self, cost: CostModel, arms: Sequence[CompressionConfig] | None = None,
                 gamma_max: int = 8, decay: float = 0.995, min_speedup: float = 1.05,
                 switch_amortize: int = 32, commit_rounds: int = 1, seed: int = 0,
                 prior: tuple[float, float] = (2.0, 1.0)) -> None:
        self.cost = cost
        self.arms = list(arms or default_arms())
        self.gamma_max = gamma_max
        self.decay = decay
        self.min_speedup = min_speedup
        self.switch_amortize = max(1, switch_amortize)
        self.commit_rounds = max(1, commit_rounds)
        self._held: CompressionConfig | None = None
        self._since_switch = 0
        self.switches = 0
        self.rng = np.random.default_rng(seed)
        self.prior = prior
        self.post: dict = {}
        self.n_decisions = 0

    def _beta(self, cfg, key) -> _Beta:
        b = self.post.get((key, cfg))
        if b is None:
            b = self.post[(key, cfg)] = _Beta(*self.prior)
        return b

    def select(self, ctx: int, key: str | None = None):
        self.n_decisions += 1
        self._since_switch += 1
        base = 1.0 / self.cost.t_baseline(ctx)
        if self._held is not None:
            a_held = self._beta(self._held, key).sample(self.rng)
            g_held, t_held = best_gamma(self.cost, self._held, a_held, ctx, self.gamma_max)
            if self._since_switch < self.commit_rounds:
                if g_held > 0 and t_held >= base * self.min_speedup:
                    return self._held, g_held
                if g_held == 0:
                    return self._held, 0
        penalty = self.cost.rebuild_cost(ctx) / self.switch_amortize
        pick, pick_g, pick_t = self.arms[0], 0, base
        for cfg in self.arms:
            a = self._beta(cfg, key).sample(self.rng)
            g, t = best_gamma(self.cost, cfg, a, ctx, self.gamma_max,
                              0.0 if cfg == self._held else penalty)
            if g > 0 and t > pick_t:
                pick, pick_g, pick_t = cfg, g, t
        if pick_g > 0 and pick != self._held:
            self._held, self._since_switch = pick, 0
            self.switches += 1
        if pick_g > 0 and pick_t < base * self.min_speedup:
            pick_g = 0
        return pick, pick_g

    def update(self, cfg, gamma, accepted, ctx, key=None) -> None:
        if gamma > 0:
            self._beta(cfg, key).observe(accepted, gamma, self.decay)

    def alpha_estimates(self, key: str | None = None) -> dict:
        return {c: self._beta(c, key).mean for c in self.arms}

    def best_known(self, ctx: int, key: str | None = None):
        best = None
        for cfg in self.arms:
            g, t = best_gamma(self.cost, cfg, self._beta(cfg, key).mean, ctx, self.gamma_max)
            if best is None or (t, cfg) > (best[0], best[1]):
                best = (t, cfg, g)
        t, cfg, g = best
        return cfg, g, t


class FlatBandit:
    """Every (config, gamma) pair as its own arm (controller.py:173-210)."""

    def __init__(self, cost: CostModel, arms: Sequence[CompressionConfig] | None = None,
                 gamma_max: int = 8, decay: float = 0.995, seed: int = 0) -> None:
        self.cost = cost
        self.cfgs = list(arms or default_arms())
        self.gamma_max = gamma_max
        self.decay = decay
        self.rng = np.random.default_rng(seed)
        self.post = {(c, g): _Beta(2.0, 1.0) for c in self.cfgs for g in range(1, gamma_max + 1)}

    def select(self, ctx: int, key: str | None = None):
        best, best_t = (self.cfgs[0], 1), -1.0
        for (cfg, g), post in self.post.items():
            t = self.cost.throughput(cfg, g, post.sample(self.rng), ctx)
            if t > best_t:
                best, best_t = (cfg, g), t
        return best

    def update(self, cfg, gamma, accepted, ctx, key=None) -> None:
        if gamma > 0:
            self.post[(cfg, gamma)].observe(accepted, gamma, self.decay)


class OraclePolicy:
    """Plays the exact argmax given every arm's true alpha (controller.py:213-230)."""

    def __init__(self, cost: CostModel, alphas: dict, gamma_max: int = 8) -> None:
        self.cost = cost
        self.alphas = alphas
        self.gamma_max = gamma_max

    def select(self, ctx: int, key: str | None = None):
        best = None
        for cfg, a in self.alphas.items():
            g, t = best_gamma(self.cost, cfg, a, ctx, self.gamma_max)
            if best is None or (t, cfg) > (best[0], best[1]):
                best = (t, cfg, g)
        return best[1], best[2]

    def update(self, cfg, gamma, accepted, ctx, key=None) -> None:
        return None


class DepthThompsonController:
    """Thompson sampling with one Beta per (config, draft depth); depths with
    too few observations reuse the deepest observed draw (controller.py:233-335)."""

    def __init__(self, cost: CostModel, arms: Sequence[CompressionConfig] | None = None,
                 gamma_max: int = 12, decay: float = 0.995, min_speedup: float = 1.05,
                 switch_amortize: int = 32, seed: int = 0,
                 prior: tuple[float, float] = (2.0, 1.0), min_obs: float = 1.0) -> None:
        self.cost = cost
        self.arms = list(arms or default_arms())
        self.gamma_max = gamma_max
        self.decay = decay
        self.min_speedup = min_speedup
        self.switch_amortize = max(1, switch_amortize)
        self.rng = np.random.default_rng(seed)
        self.prior = prior
        self.min_obs = min_obs
        self.post: dict = {}
        self.obs: dict = {}
        self._held = None
        self.switches = 0

    def _profile_post(self, cfg, key):
        k = (key, cfg)
        if k not in self.post:
            self.post[k] = [_Beta(*self.prior) for _ in range(self.gamma_max)]
            self.obs[k] = [0.0] * self.gamma_max
        return self.post[k]

    def sample_profile(self, cfg, key=None) -> list[float]:
        post = self._profile_post(cfg, key)
        obs = self.obs[(key, cfg)]
        prof, last = [], None
        for d in range(self.gamma_max):
            if obs[d] >= self.min_obs:
                last = post[d].sample(self.rng)
                prof.append(last)
            elif last is not None:
                prof.append(last)
            else:
                prof.append(post[d].sample(self.rng))
        return prof

    def mean_profile(self, cfg, key=None) -> list[float]:
        post = self._profile_post(cfg, key)
        obs = self.obs[(key, cfg)]
        prof, last = [], None
        for d in range(self.gamma_max):
            if obs[d] >= self.min_obs:
                last = post[d].mean
            prof.append(last if last is not None else post[d].mean)
        return prof

    def select(self, ctx: int, key: str | None = None):
        base = 1.0 / self.cost.t_baseline(ctx)
        penalty = self.cost.rebuild_cost(ctx) / self.switch_amortize
        pick, pick_g, pick_t = self.arms[0], 0, base
        for cfg in self.arms:
            prof = self.sample_profile(cfg, key)
            g, t = best_gamma_profile(self.cost, cfg, prof, ctx,
                                      0.0 if cfg == self._held else penalty)
            if g > 0 and t > pick_t:
                pick, pick_g, pick_t = cfg, g, t
        if pick_g > 0 and pick != self._held:
            self._held = pick
            self.switches += 1
        if pick_g > 0 and pick_t < base * self.min_speedup:
            pick_g = 0
        return pick, pick_g

    def update(self, cfg, gamma, accepted, ctx, key=None) -> None:
        if gamma <= 0:
            return
        post = self._profile_post(cfg, key)
        obs = self.obs[(key, cfg)]
        for d in range(min(accepted, self.gamma_max)):
            post[d].observe(1, 1, self.decay)
            obs[d] += 1
        if accepted < gamma and accepted < self.gamma_max:
            post[accepted].observe(0, 1, self.decay)
            obs[accepted] += 1
