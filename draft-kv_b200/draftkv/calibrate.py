"""CostModel constants measured on the device (reference throughput.py:77-81).

The reference's CostModel prices a round from bytes moved at `bandwidth`
plus fixed constants whose defaults describe an H100-class device:
fixed_draft (launch and sampling overhead of a draft step), fixed_verify (of
a verify pass) and resync_per_token (rewriting one accepted position into the
drafter cache, also the cost of a configuration switch).
`calibrate_cost_model` fits them to CUDA-event timings of this device's own
rounds, so that `select()` gates drafting with the device's real costs:

  bandwidth    = bytes of a verify pass (weights + full KV) / measured time:
                 the device's effective rate (its kernels reach a fraction
                 of the copy peak, and that fraction multiplies every byte);
  fixed_verify = 0 (the verify pass defines the rate);
  fixed_draft  = measured draft step - (weights + drafter KV) / bandwidth,
                 clamped at 0 (a drafter that streams its bytes faster than
                 the verify pass is priced at the verify pass's rate);
  compute_per_token = 0 (the measured times include the arithmetic);
  resync_per_token  = measured resync of a round / tokens emitted per sequence
  rebuild_per_token = measured partial rebuild / (ctx x changed layers / layers)

With the full cache in host memory (full_kv_bandwidth below bandwidth) the
verify pass is priced by the host link, so there the draft step defines the
rate and fixed_verify is the verify pass's residual.  Fitting constant
offsets instead would price an arm's extra bytes at the copy peak: a 16-bit
drafter kept whole would look cheaper than the verify pass it equals.  The
draft step includes the on-device sampling and the verify pass the
acceptance kernel, as the reference's constants do.
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np

from .config import CompressionConfig
from .controller import FixedPolicy
from .throughput import CostModel


def calibrate_cost_model(session, cm: CostModel, cfg: CompressionConfig, gamma: int, rounds: int = 6,
                         rebuild_layers: int = 2) -> tuple[CostModel, dict]:
    """Runs `rounds` timed rounds of `session` at (cfg, gamma) after one
    untimed round (which builds or switches the drafter cache), then one
    partial rebuild of `rebuild_layers` layers, and returns the calibrated
    cost model and the measurements.  The session's controller is restored
    afterwards; the rounds are real decode rounds (their tokens are emitted)."""
    import torch

    eng = session.eng
    saved = eng.controller
    eng.controller = FixedPolicy(cfg, gamma)
    try:
        session.round()                          # builds / switches the drafter cache
        eng.phase_events = []
        tokens = []
        for _ in range(rounds):
            out = session.round()
            tokens += [k + 1 for k, _e in out]
        ev, eng.phase_events = eng.phase_events, None
        # a partial rebuild at the current context (same configuration: the
        # rebuilt layers restart at zero eviction scores, outputs unchanged)
        st = session.st
        ctx = min(len(t) for t in session.toks) - 1
        n_l = max(1, min(rebuild_layers, session.m.n_layers))
        ctx_t = torch.tensor([len(t) - 1 for t in session.toks], dtype=torch.int32, device=session.m.device)
        eng.rebuild_events = []
        eng._rebuild(st, list(range(n_l)), ctx_t, advance=False)
        rb, eng.rebuild_events = eng.rebuild_events, None
        torch.cuda.synchronize()
    finally:
        eng.controller = saved
        eng.phase_events = None
        eng.rebuild_events = None
    draft = [e[0].elapsed_time(e[1]) * 1e-3 / g for g, e in ev if g > 0]
    verify = [e[1].elapsed_time(e[2]) * 1e-3 for g, e in ev if g > 0]
    resync = [e[2].elapsed_time(e[3]) * 1e-3 for g, e in ev if g > 0]
    if not draft:
        raise RuntimeError("calibration rounds did not draft (gamma clamped to 0 near the end of generation)")
    t_rebuild = rb[0][1].elapsed_time(rb[0][2]) * 1e-3 if rb else 0.0
    return fit_constants(cm, cfg, gamma, ctx, float(np.median(draft)), float(np.median(verify)),
                         float(np.median(resync)), t_rebuild, n_l, float(np.mean(tokens)) if tokens else 1.0)


def fit_constants(cm: CostModel, cfg, gamma: int, ctx: int, t_draft: float, t_verify: float, t_resync: float,
                  t_rebuild: float, rebuild_layers: int, tokens_per_round: float) -> tuple[CostModel, dict]:
    """The calibrated cost model from measured seconds (see the module
    docstring): a draft step, a (gamma+1)-token verify pass, the resync of a
    round that emitted `tokens_per_round` tokens per sequence, and a rebuild
    of `rebuild_layers` layers at context ctx."""
    b_draft = cm.weight_bytes + cm.draft_kv_bytes(cfg, ctx)
    b_kv = cm.full_kv_bytes(ctx)
    if cm.full_kv_bandwidth < cm.bandwidth:      # full cache over the host link
        bw = b_draft / max(t_draft, 1e-12)
        fixed_draft = 0.0
        fixed_verify = max(0.0, t_verify - cm.weight_bytes / bw - b_kv / cm.full_kv_bandwidth)
        full_bw = cm.full_kv_bandwidth
    else:
        bw = (cm.weight_bytes + b_kv) / max(t_verify, 1e-12)
        fixed_verify = 0.0
        fixed_draft = max(0.0, t_draft - b_draft / bw)
        full_bw = bw
    resync_per_token = max(0.0, t_resync) / max(tokens_per_round, 1e-9)
    rebuild_per_token = (t_rebuild / (ctx * rebuild_layers / cm.n_layers)
                         if t_rebuild > 0 and ctx > 0 and rebuild_layers > 0 else None)
    out = replace(cm, bandwidth=bw, full_kv_bandwidth=full_bw, compute_per_token=0.0, fixed_draft=fixed_draft,
                  fixed_verify=fixed_verify, resync_per_token=resync_per_token, rebuild_per_token=rebuild_per_token)
    meas = dict(cfg=cfg.label(), gamma=gamma, ctx=ctx, t_draft_step_s=t_draft, t_verify_s=t_verify,
                bandwidth=bw, copy_peak=cm.bandwidth,
                t_resync_s=t_resync, t_rebuild_s=t_rebuild, rebuild_layers=rebuild_layers,
                tokens_per_round=tokens_per_round, fixed_draft=fixed_draft, fixed_verify=fixed_verify,
                resync_per_token=resync_per_token, rebuild_per_token=rebuild_per_token)
    return out, meas
