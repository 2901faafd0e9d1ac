"""Multi-process decoding: sequences shard by rank, the controller is replicated.

Every process runs its own engine over its own sequences (weak scaling, no
tensor or sequence parallelism).  The only data that crosses processes are
the controller's inputs -- each sequence's (accepted, context, gamma) per
round -- and, at the end, the emitted token ids.  Every process feeds the
same gathered records, in the same order, to an identically seeded
controller, so all controllers make the same decisions without a broadcast.

`ControllerExchange` (used by `Session.round` when given) ships the records
in batches: each process buffers its records for `period` rounds, then one
asynchronous all-gather (NCCL on CUDA tensors across GPUs, gloo on CPU
tensors) carries every process's batch; every process applies the batch
`lag` rounds later, rounds in order, processes in rank order, sequences in
order, and selects on the largest context known from the applied records.
The collective runs on the communication library's stream while the next
rounds compute, and ranks are not held in step every round: a process waits
only when a batch it must apply has not arrived.  Feedback reaches the
controller up to period + lag rounds late (the same delay on every process).

`allgather_exchange` + `replicated_select` / `replicated_update` is the
per-round, blocking form of the same protocol (used by the CPU tests and by
callers that want the reference's undelayed feedback).
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


class ControllerExchange:
    """Batched, asynchronous replication of the controller's inputs (see the
    module docstring).  One instance per process and session; every process
    must call start() once, then select() and update() once per round in
    the same order, then finish()."""

    def __init__(self, max_records: int, period: int = 8, lag: int = 2, group=None, device=None) -> None:
        import torch.distributed as dist
        self.max_records = int(max_records)
        self.period = max(1, int(period))
        self.lag = max(1, int(lag))     # 1: applied at the very next select (no overlap)
        self.group = group
        self.device = device
        self.world = dist.get_world_size(group)
        self.round = 0
        self.ctx = 0
        self._cfgs: list = []          # the configuration selected in each round (equal on every process)
        self._buf: list = []           # this process's records of the rounds not shipped yet
        self._pending: list = []       # (due round, first round, n rounds, work, output)
        self.applied = 0
        self.batches = 0

    def _gather(self, rows, async_op: bool):
        import torch
        import torch.distributed as dist
        t = torch.tensor(rows, dtype=torch.int64, device=self.device)
        # output concatenated along the first dimension (both backends take it)
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=torch.int64, device=self.device)
        work = dist.all_gather_into_tensor(out, t, group=self.group, async_op=async_op)
        return work, out.view((self.world,) + tuple(t.shape))

    def start(self, local_ctx: int) -> None:
        """One blocking exchange of the processes' starting contexts."""
        work, out = self._gather([int(local_ctx)], async_op=False)
        self.ctx = int(out.max().item())

    def _apply(self, controller, key, limit: int) -> None:
        while self._pending and self._pending[0][0] <= limit:
            _due, r0, n, work, out = self._pending.pop(0)
            work.wait()
            rows = out.cpu().tolist()              # [world][n][max_records][4]
            for j in range(n):
                cfg = self._cfgs[r0 + j]
                for p in range(self.world):
                    for k, c, g, nxt in rows[p][j]:
                        if c < 0:
                            continue
                        self.ctx = max(self.ctx, nxt)
                        if k >= 0:
                            controller.update(cfg, g, k, c, key)
                            self.applied += 1

    def select(self, controller, key=None):
        """Applies the batches due by this round, then selects on the largest
        context they report."""
        self._apply(controller, key, self.round)
        cfg, gamma = controller.select(self.ctx, key)
        self._cfgs.append(cfg)
        return cfg, gamma

    def update(self, records: Sequence[tuple]) -> None:
        """This round's records (accepted, context, gamma, next context) of
        this process's sequences (accepted < 0: context only); ships the batch
        at the end of a period."""
        if len(records) > self.max_records:
            raise ValueError(f"{len(records)} records > max_records {self.max_records}")
        rows = [[int(k), int(c), int(g), int(n)] for k, c, g, n in records]
        rows += [[-1, -1, -1, -1]] * (self.max_records - len(rows))
        self._buf.append(rows)
        self.round += 1
        if len(self._buf) == self.period:
            self._ship()

    def _ship(self) -> None:
        n = len(self._buf)
        work, out = self._gather(self._buf, async_op=True)
        self._pending.append((self.round + self.lag - 1, self.round - n, n, work, out))
        self._buf = []
        self.batches += 1

    def finish(self, controller, key=None) -> None:
        """Ships a partial batch and applies everything outstanding."""
        if self._buf:
            self._ship()
        self._apply(controller, key, float("inf"))


def gather_tokens(sequences: Sequence[Sequence[int]], group=None) -> list:
    """Every process's token lists, concatenated in rank order (the
    end-of-run gather of the emitted streams)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    out = [None] * world
    dist.all_gather_object(out, [list(map(int, s)) for s in sequences], group=group)
    return [s for part in out for s in part]
