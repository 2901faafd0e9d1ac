"""Tokens per verify pass and the memory-traffic cost model.

Same functions and the same formulas as the reference's
draftkv/throughput.py:24-268: `expected_tokens`, `expected_tokens_profile`,
`CostModel` (t_draft / t_verify / t_baseline / rebuild_cost / throughput /
speedup / ceiling) and the gamma scans `best_gamma`, `best_gamma_profile`.
The B200 build instantiates CostModel with measured numbers (HBM bandwidth,
exact weight bytes, sequences per GPU) and reports speedup against
`ceiling()`.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

from .config import CompressionConfig


def _clip01(a: float) -> float:
    return min(1.0, max(0.0, float(a)))


def expected_tokens(alpha: float, gamma: int) -> float:
    """E = (1 - a^(g+1)) / (1 - a): accepted run plus the bonus token
    (throughput.py:24-38)."""
    a = _clip01(alpha)
    if gamma < 0:
        raise ValueError("gamma must be >= 0")
    if a >= 1.0 - 1e-12:
        return float(gamma + 1)
    return float((1.0 - a ** (gamma + 1)) / (1.0 - a))


def expected_tokens_profile(accept: Sequence[float]) -> float:
    """E = 1 + sum_k prod_{i<k} a_i for a depth-indexed profile (throughput.py:41-56)."""
    tot, run = 1.0, 1.0
    for a in accept:
        run *= _clip01(a)
        tot += run
    return tot


@dataclass
class CostModel:
    """Per-round wall-clock model built from bytes moved (throughput.py:59-225).

    Drafting and verifying run the same weights, so every byte saved is a KV
    byte; `ceiling()` is the speedup as alpha -> 1 and gamma -> infinity.
    """

    n_layers: int = 32
    n_kv_heads: int = 8
    d_head: int = 128
    weight_bytes: float = 16.0e9
    bandwidth: float = 2.0e12
    full_kv_bandwidth: float | None = None
    batch: int = 1
    hbm_kv_budget: float | None = None
    compute_per_token: float = 1.0e-6
    fixed_draft: float = 5.0e-6
    fixed_verify: float = 1.0e-5
    resync_per_token: float = 2.0e-6
    controller_overhead: float = 1.0e-6
    # Seconds to re-derive one context position of every layer of the
    # drafter cache on a configuration switch.  None: resync_per_token, as
    # in the reference; a cost model calibrated on the device (calibrate.py)
    # sets it from a timed partial rebuild, since the device's per-round
    # resync and its bulk rebuild run at very different rates per position.
    rebuild_per_token: float | None = None

    def __post_init__(self) -> None:
        if self.full_kv_bandwidth is None:
            self.full_kv_bandwidth = self.bandwidth

    # ------------------------------------------------------------- bytes
    def full_kv_bytes(self, ctx: int) -> float:
        return 2.0 * ctx * self.n_layers * self.n_kv_heads * self.d_head * 2.0 * self.batch

    def draft_kv_bytes(self, cfg, ctx: int) -> float:
        if hasattr(cfg, "per_layer_bytes"):
            return cfg.per_layer_bytes(ctx, self.n_kv_heads, self.d_head) * self.batch
        kept = min(ctx, max(cfg.sink + cfg.recent, int(round(cfg.keep_frac * ctx))))
        return (2.0 * kept * self.n_layers * self.n_kv_heads
                * cfg.bytes_per_entry(self.d_head) * self.batch)

    # ------------------------------------------------------------- times
    def _kv_read_time(self, nbytes: float) -> float:
        if self.hbm_kv_budget is None:
            return nbytes / self.bandwidth
        inside = min(nbytes, self.hbm_kv_budget)
        outside = max(0.0, nbytes - self.hbm_kv_budget)
        return inside / self.bandwidth + outside / self.full_kv_bandwidth

    def draft_kv_resident_frac(self, cfg: CompressionConfig, ctx: int) -> float:
        n = self.draft_kv_bytes(cfg, ctx)
        if self.hbm_kv_budget is None or n <= 0:
            return 1.0
        return min(1.0, self.hbm_kv_budget / n)

    def t_draft(self, cfg, ctx: int) -> float:
        return (self.weight_bytes / self.bandwidth
                + self._kv_read_time(self.draft_kv_bytes(cfg, ctx))
                + self.compute_per_token + self.fixed_draft)

    def t_verify(self, ctx: int, gamma: int) -> float:
        return (self.weight_bytes / self.bandwidth
                + self.full_kv_bytes(ctx) / self.full_kv_bandwidth
                + (gamma + 1) * self.compute_per_token + self.fixed_verify)

    def t_baseline(self, ctx: int) -> float:
        return (self.weight_bytes / self.bandwidth
                + self.full_kv_bytes(ctx) / self.full_kv_bandwidth
                + self.compute_per_token + self.fixed_verify)

    def rebuild_cost(self, ctx: int, layers_changed: int | None = None) -> float:
        nl = max(1, self.n_layers)
        frac = 1.0 if layers_changed is None else min(1.0, layers_changed / nl)
        rate = self.resync_per_token if self.rebuild_per_token is None else self.rebuild_per_token
        return ctx * rate * frac * self.n_layers / nl

    # -------------------------------------------------------- objectives
    def round_cost(self, cfg, gamma: int, alpha: float, ctx: int, extra_cost: float = 0.0) -> float:
        return (gamma * self.t_draft(cfg, ctx) + self.t_verify(ctx, gamma)
                + expected_tokens(alpha, gamma) * self.resync_per_token
                + self.controller_overhead + extra_cost)

    def throughput(self, cfg, gamma: int, alpha: float, ctx: int, extra_cost: float = 0.0) -> float:
        if gamma == 0:
            return 1.0 / self.t_baseline(ctx)
        return expected_tokens(alpha, gamma) / self.round_cost(cfg, gamma, alpha, ctx, extra_cost)

    def round_cost_profile(self, cfg, accept: Sequence[float], ctx: int, extra_cost: float = 0.0) -> float:
        g = len(accept)
        return (g * self.t_draft(cfg, ctx) + self.t_verify(ctx, g)
                + expected_tokens_profile(accept) * self.resync_per_token
                + self.controller_overhead + extra_cost)

    def throughput_profile(self, cfg, accept: Sequence[float], ctx: int, extra_cost: float = 0.0) -> float:
        if not accept:
            return 1.0 / self.t_baseline(ctx)
        return expected_tokens_profile(accept) / self.round_cost_profile(cfg, accept, ctx, extra_cost)

    def speedup(self, cfg, gamma: int, alpha: float, ctx: int) -> float:
        return self.throughput(cfg, gamma, alpha, ctx) * self.t_baseline(ctx)

    def ceiling(self, cfg, ctx: int) -> float:
        base = self.weight_bytes / self.bandwidth + self.full_kv_bytes(ctx) / self.full_kv_bandwidth
        draft = self.weight_bytes / self.bandwidth + self._kv_read_time(self.draft_kv_bytes(cfg, ctx))
        return ((base + self.compute_per_token + self.fixed_verify)
                / (draft + self.compute_per_token + self.fixed_draft + self.resync_per_token))


def best_gamma(cost: CostModel, cfg, alpha: float, ctx: int, gamma_max: int = 8,
               extra_cost: float = 0.0) -> tuple[int, float]:
    """Scan gamma = 0..gamma_max for the best throughput; 0 = do not draft
    (throughput.py:249-268)."""
    g_best, t_best = 0, cost.throughput(cfg, 0, alpha, ctx)
    for g in range(1, gamma_max + 1):
        t = cost.throughput(cfg, g, alpha, ctx, extra_cost)
        if t > t_best:
            g_best, t_best = g, t
    return g_best, t_best


def best_gamma_profile(cost: CostModel, cfg, accept: Sequence[float], ctx: int,
                       extra_cost: float = 0.0) -> tuple[int, float]:
    """Full scan over prefixes of a depth profile (throughput.py:228-246)."""
    g_best, t_best = 0, cost.throughput_profile(cfg, (), ctx)
    for g in range(1, len(accept) + 1):
        t = cost.throughput_profile(cfg, accept[:g], ctx, extra_cost)
        if t > t_best:
            g_best, t_best = g, t
    return g_best, t_best
