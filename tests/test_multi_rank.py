"""Multi-process decoding on CPU (gloo, world size 2): the per-round exchange
of draftkv.dist keeps replicated, identically seeded controllers identical
although each process holds different sequences (contexts, acceptances and,
near the end of generation, clamped gammas)."""
import json
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROUNDS = 40


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "draft-kv_b200")]
    from draftkv import CostModel, ThompsonController, default_arms
    from draftkv.dist import allgather_exchange, replicated_select, replicated_update

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cm = CostModel(n_layers=32, n_kv_heads=8, d_head=128, weight_bytes=15.0e9, bandwidth=6.5e12, batch=4)
        ctrl = ThompsonController(cm, default_arms(), gamma_max=8, seed=0)
        ex = allgather_exchange(4)
        rng = np.random.default_rng(100 + rank)               # each process: its own sequences
        ctx = [2000 + 300 * rank + 7 * b for b in range(4)]
        decisions = []
        for r in range(ROUNDS):
            cfg, gamma = replicated_select(ctrl, max(ctx), None, ex)
            g_local = min(gamma, 2) if (rank == 1 and r % 5 == 4) else gamma   # a clamped gamma
            if g_local == 0:
                recs = []
            else:
                recs = [(int(rng.integers(0, g_local + 1)), c, g_local) for c in ctx]
            applied = replicated_update(ctrl, cfg, recs, None, ex)
            for i, (k, _c, g) in enumerate(recs):
                ctx[i] += k + 1
            decisions.append([cfg.label(), int(gamma), len(applied)])
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(decisions, f)
    finally:
        dist.destroy_process_group()


def test_replicated_controllers_agree_over_gloo(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    d0 = json.loads((tmp_path / "rank0.json").read_text())
    d1 = json.loads((tmp_path / "rank1.json").read_text())
    assert len(d0) == ROUNDS
    assert d0 == d1
    # both processes' records were applied every drafting round
    assert all(n == 8 for cfg, g, n in d0 if g > 0)
    # the controller explores: more than one (config, gamma) decision
    assert len({(c, g) for c, g, _n in d0}) > 1


def test_exchange_without_processes_is_local():
    """Without an exchange the two steps use the local context and records."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.join(os.path.dirname(here), "draft-kv_b200")]
    from draftkv import CostModel, ThompsonController, default_arms
    from draftkv.dist import replicated_select, replicated_update

    cm = CostModel(n_layers=32, n_kv_heads=8, d_head=128, weight_bytes=15.0e9, bandwidth=6.5e12, batch=4)
    a = ThompsonController(cm, default_arms(), gamma_max=8, seed=3)
    b = ThompsonController(cm, default_arms(), gamma_max=8, seed=3)
    for r in range(10):
        ca, ga = replicated_select(a, 4096 + r, None, None)
        cb, gb = b.select(4096 + r, None)
        assert (ca, ga) == (cb, gb)
        recs = [(1, 4096 + r, ga), (-1, 9999, 0)] if ga > 0 else []
        applied = replicated_update(a, ca, recs, None, None)
        for k, c, g in applied:
            b.update(cb, g, k, c, None)
        assert all(k >= 0 for k, _c, _g in applied)


def _rank_main_batched(rank: int, world: int, port: int, out_dir: str) -> None:
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "draft-kv_b200")]
    from draftkv import CostModel, ThompsonController, default_arms
    from draftkv.dist import ControllerExchange, gather_tokens

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cm = CostModel(n_layers=32, n_kv_heads=8, d_head=128, weight_bytes=15.0e9, bandwidth=6.5e12, batch=4)
        ctrl = ThompsonController(cm, default_arms(), gamma_max=8, seed=0)
        ex = ControllerExchange(4, period=3, lag=2)
        rng = np.random.default_rng(100 + rank)
        ctx = [2000 + 300 * rank + 7 * b for b in range(4)]
        ex.start(max(ctx))
        decisions, sent = [], 0
        for r in range(ROUNDS):
            cfg, gamma = ex.select(ctrl, None)
            active = [b for b in range(4) if not (rank == 1 and b == 3 and r > 30)]   # a finished sequence
            recs = []
            for b in active:
                k = int(rng.integers(0, gamma + 1)) if gamma > 0 else -1
                step = k + 1 if gamma > 0 else 1
                recs.append((k, ctx[b], gamma, ctx[b] + step))
                ctx[b] += step
                sent += k >= 0
            ex.update(recs)
            decisions.append([cfg.label(), int(gamma), ex.ctx])
        ex.finish(ctrl, None)
        toks = gather_tokens([[rank, b] for b in range(2)])
        state = {f"{k}|{c.label()}": [round(v.a, 9), round(v.b, 9)] for (k, c), v in ctrl.post.items()}
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(dict(decisions=decisions, applied=ex.applied, sent=sent, tokens=toks, state=state,
                           batches=ex.batches), f)
    finally:
        dist.destroy_process_group()


def test_batched_exchange_keeps_controllers_identical_over_gloo(tmp_path):
    """The batched, asynchronous exchange: identical decisions and identical
    final posteriors on both processes, every process's records applied on
    every process, feedback applied lag rounds after each batch, and the
    end-of-run token gather in rank order."""
    world = 2
    mp.start_processes(_rank_main_batched, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    r0 = json.loads((tmp_path / "rank0.json").read_text())
    r1 = json.loads((tmp_path / "rank1.json").read_text())
    assert r0["decisions"] == r1["decisions"] and len(r0["decisions"]) == ROUNDS
    assert r0["state"] == r1["state"]
    assert r0["applied"] == r1["applied"] == r0["sent"] + r1["sent"]
    assert r0["batches"] == -(-ROUNDS // 3)
    # the first batch (rounds 0-2) is applied at round 4 (its last round + lag 2)
    assert all(d[2] == r0["decisions"][0][2] for d in r0["decisions"][:4])
    assert r0["decisions"][4][2] > r0["decisions"][0][2]
    assert r0["tokens"] == r1["tokens"] == [[0, 0], [0, 1], [1, 0], [1, 1]]
    assert len({(c, g) for c, g, _x in r0["decisions"]}) > 1
