"""The draft/verify loop, restated (test infrastructure only).

Follows draftkv/engine.py:25-223.  Invariant (engine.py:3-12): the caches hold
positions 0 .. len(tokens)-2 and tokens[-1] is pending, never cached, so the
verify block is [tokens[-1]] + drafts at start_pos = n-1.

Random numbers come from one numpy Generator consumed in the reference's order
(a draw per drafted token even under greedy decoding, engine.py:178), so token
streams under sampling reproduce the reference exactly.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .caches import OracleComp, OracleFull


def probs_of(logits, temperature):
    """engine.py:36-42: one-hot at the first argmax for T <= 0, else fp64
    softmax(logits / T)."""
    if temperature <= 0.0:
        p = np.zeros(logits.shape, np.float64)
        p[int(np.argmax(logits))] = 1.0
        return p
    z = logits.astype(np.float64) / temperature
    z = z - z.max()
    e = np.exp(z)
    return e / e.sum()


@dataclass
class OracleRound:
    cfg: object
    gamma: int
    accepted: int
    emitted: int
    ctx: int


@dataclass
class OracleResult:
    tokens: list
    rounds: list = field(default_factory=list)
    draft_steps: int = 0
    verify_passes: int = 0
    cache_rebuilds: int = 0
    layers_rebuilt: int = 0


class OracleEngine:
    def __init__(self, model, controller, seed=0, full_factory=None):
        self.model = model
        self.controller = controller
        self.rng = np.random.default_rng(seed)
        self.full_factory = full_factory or (lambda: OracleFull(model.n_layers))

    def _draw(self, p):
        """engine.py:101-106."""
        p = np.clip(p, 0.0, None)
        tot = p.sum()
        if tot <= 0:
            return int(self.rng.integers(len(p)))
        return int(self.rng.choice(len(p), p=p / tot))

    def generate_baseline(self, prompt, max_new, temperature=0.0):
        """engine.py:109-120."""
        toks = list(prompt)
        cache = self.full_factory()
        if len(toks) > 1:
            self.model.forward(np.array(toks[:-1]), cache, 0)
        for _ in range(max_new):
            lg = self.model.forward(np.array([toks[-1]]), cache, len(toks) - 1)[-1]
            toks.append(self._draw(probs_of(lg, temperature)))
        return toks

    def generate(self, prompt, max_new, temperature=0.0, key=None):
        """engine.py:123-223."""
        m = self.model
        toks = list(prompt)
        full = self.full_factory()
        if len(toks) > 1:
            m.forward(np.array(toks[:-1]), full, 0)
        comp, comp_cfg = None, None
        res = OracleResult(tokens=toks)
        while len(toks) - len(prompt) < max_new:
            n = len(toks)
            left = max_new - (n - len(prompt))
            cfg, gamma = self.controller.select(n, key)
            gamma = min(gamma, max(left - 1, 0))
            if gamma <= 0:
                lg = m.forward(np.array([toks[-1]]), full, n - 1)[-1]
                toks.append(self._draw(probs_of(lg, temperature)))
                res.verify_passes += 1
                res.rounds.append(OracleRound(cfg, 0, 0, 1, n))
                if comp is not None:
                    comp.sync_from(full, n - 1)
                continue
            if comp is None:
                comp = OracleComp(m.n_layers, cfg)
                comp.sync_from(full, 0)
                comp_cfg = cfg
                res.cache_rebuilds += 1
            elif comp_cfg != cfg:
                old = list(comp_cfg.cfgs) if hasattr(comp_cfg, "cfgs") else [comp_cfg] * m.n_layers
                new = list(cfg.cfgs) if hasattr(cfg, "cfgs") else [cfg] * m.n_layers
                changed = [L for L in range(m.n_layers) if old[L] != new[L]]
                comp.rebuild_layers(full, changed, new)
                comp_cfg = cfg
                res.cache_rebuilds += 1
                res.layers_rebuilt += len(changed)
            drafts, dprobs = [], []
            x = toks[-1]
            for i in range(gamma):
                lg = m.forward(np.array([x]), comp, n - 1 + i)[-1]
                q = probs_of(lg, temperature)
                x = self._draw(q)
                drafts.append(x)
                dprobs.append(q)
            res.draft_steps += gamma
            lg = m.forward(np.array([toks[-1]] + drafts), full, n - 1)
            res.verify_passes += 1
            k = 0
            for i in range(gamma):
                if temperature <= 0.0:
                    ok = int(np.argmax(lg[i])) == drafts[i]
                else:
                    p = probs_of(lg[i], temperature)
                    qd = dprobs[i][drafts[i]]
                    ok = self.rng.random() < min(1.0, p[drafts[i]] / qd if qd > 0 else 0.0)
                if not ok:
                    break
                k += 1
            out = drafts[:k]
            if k == gamma:
                nxt = self._draw(probs_of(lg[gamma], temperature))
            elif temperature <= 0.0:
                nxt = int(np.argmax(lg[k]))
            else:
                p = probs_of(lg[k], temperature)
                r = np.clip(p - dprobs[k], 0.0, None)
                nxt = self._draw(r if r.sum() > 0 else p)
            out.append(nxt)
            toks.extend(out)
            full.truncate(n + k)
            comp.sync_from(full, n - 1)
            self.controller.update(cfg, gamma, k, n, key)
            res.rounds.append(OracleRound(cfg, gamma, k, len(out), n))
        res.tokens = toks
        return res
