"""Multi-process decoding: sequences shard by rank, the controller is replicated.

Every process runs its own engine over its own sequences (weak scaling, no
tensor or sequence parallelism).  The only data that crosses processes are the
per-round controller inputs: each process's largest context before `select`
and its per-sequence (accepted, context, gamma) after the round.  Every process
feeds the same gathered lists to an identically seeded controller, so all
controllers make the same decisions without a broadcast.

`allgather_exchange` builds the exchange over torch.distributed (NCCL on
CUDA tensors across GPUs, gloo on CPU tensors); `replicated_select` and
`replicated_update` are the two steps of a round, used by `Session.round`.
Every process must take part in both steps of every round, in the same order.
"""

from __future__ import annotations

from typing import Callable, Optional, Sequence

Record = tuple          # (accepted, context, gamma); accepted < 0 marks a context-only record
Exchange = Callable[[Sequence[Record]], list]


def allgather_exchange(max_records: int, group=None, device=None) -> Exchange:
    """An exchange over torch.distributed.all_gather: each process passes at
    most `max_records` records; every process receives all records of all
    processes in rank order."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)

    def exchange(records: Sequence[Record]) -> list:
        if len(records) > max_records:
            raise ValueError(f"{len(records)} records > max_records {max_records}")
        rows = [[int(k), int(c), int(g)] for k, c, g in records]
        rows += [[-1, -1, -1]] * (max_records - len(rows))
        t = torch.tensor(rows, dtype=torch.int64, device=device)
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t, group=group)
        return [(k, c, g) for r in torch.stack(out).cpu().tolist() for k, c, g in r if c >= 0]

    return exchange


def replicated_select(controller, local_ctx: int, key=None, exchange: Optional[Exchange] = None):
    """controller.select on the largest context over every process (the local
    one without an exchange), so replicated controllers agree."""
    ctx = local_ctx
    if exchange is not None:
        ctx = max(c for _k, c, _g in exchange([(-1, local_ctx, 0)]))
    return controller.select(ctx, key)


def replicated_update(controller, cfg, records: Sequence[Record], key=None,
                      exchange: Optional[Exchange] = None) -> list:
    """controller.update for every (accepted, context, gamma) record of every
    process, in rank order; context-only records (accepted < 0) are skipped.
    Returns the records applied."""
    allr = list(records) if exchange is None else exchange(records)
    applied = []
    for k, ctx, g in allr:
        if k < 0:
            continue
        controller.update(cfg, g, k, ctx, key)
        applied.append((k, ctx, g))
    return applied
