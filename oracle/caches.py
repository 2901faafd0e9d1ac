"""Cache semantics of the reference, restated (test infrastructure only).

OracleFull   -- draftkv/compress.py:49-92   (exact cache, positions in order)
OracleComp   -- draftkv/compress.py:95-241  (quantized mirror with sink +
                recent + heavy-hitter eviction, resync and partial rebuild)
OraclePool   -- draftkv/paged.py:33-74      (fixed block pool, LIFO free list)
OraclePaged  -- draftkv/paged.py:76-177     (per-layer block tables, rollback
                frees whole blocks and keeps the partial tail)

Entries of one layer are kept as parallel python lists in position order,
which is the order the reference keeps them in (appends arrive in increasing
position; truncation removes a suffix).
"""

from __future__ import annotations

import numpy as np

from .quant import quantize


class OracleFull:
    """Exact cache (compress.py:49-92)."""

    def __init__(self, n_layers: int) -> None:
        self.n_layers = n_layers
        self.rows = [[] for _ in range(n_layers)]     # (k, v, pos) per entry

    def append(self, layer, k, v, pos):
        for i in range(k.shape[0]):
            self.rows[layer].append((k[i], v[i], int(pos[i])))

    def read(self, layer):
        r = self.rows[layer]
        if not r:
            return (np.zeros((0, 0, 0), np.float32), np.zeros((0, 0, 0), np.float32),
                    np.zeros((0,), np.int64))
        return (np.stack([e[0] for e in r]), np.stack([e[1] for e in r]),
                np.asarray([e[2] for e in r], np.int64))

    def note_attention(self, layer, probs):
        return None

    def truncate(self, n_pos):
        for L in range(self.n_layers):
            self.rows[L] = [e for e in self.rows[L] if e[2] < n_pos]

    @property
    def length(self):
        return len(self.rows[0])


class OracleComp:
    """Drafter cache (compress.py:95-241).

    Per layer: quantized K, V, position and accumulated attention mass.
    `seen` is the logical context length including evicted tokens; it is
    advanced by layer-0 appends and clipped by truncation (:119, :131-132, :188).
    """

    def __init__(self, n_layers, cfgs):
        if hasattr(cfgs, "cfgs"):
            cfgs = list(cfgs.cfgs)
        elif not isinstance(cfgs, (list, tuple)):
            cfgs = [cfgs] * n_layers
        if len(cfgs) != n_layers:
            raise ValueError(f"expected {n_layers} per-layer configs, got {len(cfgs)}")
        self.n_layers = n_layers
        self.cfgs = list(cfgs)
        self.k = [[] for _ in range(n_layers)]
        self.v = [[] for _ in range(n_layers)]
        self.pos = [[] for _ in range(n_layers)]
        self.score = [[] for _ in range(n_layers)]
        self.seen = 0

    # ------------------------------------------------------------ protocol
    def append(self, layer, k, v, pos):
        """compress.py:122-133: quantize, add with score 0, then evict once."""
        c = self.cfgs[layer]
        kq, vq = quantize(k, c.bits), quantize(v, c.bits)
        for i in range(kq.shape[0]):
            self.k[layer].append(kq[i])
            self.v[layer].append(vq[i])
            self.pos[layer].append(int(pos[i]))
            self.score[layer].append(0.0)
        if layer == 0:
            self.seen = max(self.seen, int(pos[-1]) + 1)
        self.evict(layer)

    def read(self, layer):
        if not self.k[layer]:
            return (np.zeros((0, 0, 0), np.float32), np.zeros((0, 0, 0), np.float32),
                    np.zeros((0,), np.int64))
        return (np.stack(self.k[layer]), np.stack(self.v[layer]),
                np.asarray(self.pos[layer], np.int64))

    def note_attention(self, layer, probs):
        """compress.py:144-151: add the (query, head)-summed mass per entry."""
        if probs.size == 0:
            return
        mass = probs.sum(axis=(0, 1))
        for i in range(min(len(self.score[layer]), mass.shape[0])):
            self.score[layer][i] += float(mass[i])

    # ------------------------------------------------------------- policy
    def budget(self, layer=0):
        """compress.py:154-157 (python round(): half to even)."""
        c = self.cfgs[layer]
        return max(int(round(c.keep_frac * max(self.seen, 1))), c.sink + c.recent)

    def evict_plan(self, layer):
        """Indices (into the layer's lists) to drop; compress.py:159-179.

        Protected: the `sink` lowest and the `recent` highest positions.  The
        reference slices the position argsort with [-recent:], so recent == 0
        protects every entry; that is reproduced.  Among the rest, the lowest
        accumulated mass goes first, ties broken by list order (= position).
        """
        c = self.cfgs[layer]
        n = len(self.pos[layer])
        budget = self.budget(layer)
        if n <= budget:
            return []
        by_pos = sorted(range(n), key=lambda i: self.pos[layer][i])
        guard = set(by_pos[: c.sink])
        guard |= set(by_pos[max(0, n - c.recent):] if c.recent > 0 else by_pos)
        cand = [i for i in range(n) if i not in guard]
        n_drop = n - budget
        if n_drop <= 0 or not cand:
            return []
        cand.sort(key=lambda i: self.score[layer][i])       # stable
        return sorted(cand[:n_drop])

    def evict(self, layer):
        drop = set(self.evict_plan(layer))
        if drop:
            self._keep(layer, [i for i in range(len(self.pos[layer])) if i not in drop])

    def _keep(self, L, idx):
        self.k[L] = [self.k[L][i] for i in idx]
        self.v[L] = [self.v[L][i] for i in idx]
        self.pos[L] = [self.pos[L][i] for i in idx]
        self.score[L] = [self.score[L][i] for i in idx]

    # ------------------------------------------------------------ control
    def truncate(self, n_pos):
        """compress.py:181-188."""
        for L in range(self.n_layers):
            self._keep(L, [i for i, p in enumerate(self.pos[L]) if p < n_pos])
        self.seen = min(self.seen, n_pos)

    def sync_from(self, full, start_pos):
        """compress.py:190-207: drop >= start_pos, re-append the true rows."""
        self.truncate(start_pos)
        rows = 0
        for L in range(self.n_layers):
            k, v, pos = full.read(L)
            sel = np.nonzero(pos >= start_pos)[0]
            if sel.size:
                self.append(L, k[sel], v[sel], pos[sel])
                rows += int(sel.size)
        return rows

    def rebuild_layers(self, full, layers, cfgs=None):
        """compress.py:209-230: clear and requantize only the named layers."""
        rows = 0
        for L in layers:
            if cfgs is not None:
                self.cfgs[L] = cfgs[L]
            self._keep(L, [])
            k, v, pos = full.read(L)
            if pos.size:
                self.append(L, k, v, pos)
                rows += int(pos.size)
        return rows

    @property
    def length(self):
        return len(self.pos[0])


class OraclePool:
    """paged.py:33-74: whole-block pool; the free list is a LIFO stack."""

    def __init__(self, n_blocks, block_size):
        self.n_blocks, self.block_size = n_blocks, block_size
        self.free_list = list(range(n_blocks))
        self.used = set()

    def allocate(self):
        if not self.free_list:
            raise RuntimeError("exhausted")
        b = self.free_list.pop()
        self.used.add(b)
        return b

    def free(self, b):
        if b not in self.used:
            raise RuntimeError(f"double free of block {b}")
        self.used.discard(b)
        self.free_list.append(b)


class OraclePaged:
    """paged.py:76-177: per-layer block tables over one shared pool."""

    def __init__(self, n_layers, n_heads, d_head, block_size=16, n_blocks=512,
                 dtype=np.float32):
        self.n_layers, self.bs = n_layers, block_size
        self.pool = OraclePool(n_blocks, block_size)
        # the store has one dtype (fp32 by default, paged.py:80-99), so rows
        # written into it are rounded to that dtype
        self.k_store = [np.zeros((n_blocks * block_size, n_heads, d_head), dtype)
                        for _ in range(n_layers)]
        self.v_store = [np.zeros_like(self.k_store[0]) for _ in range(n_layers)]
        self.table = [[] for _ in range(n_layers)]
        self.count = [0] * n_layers
        self.pos = [[] for _ in range(n_layers)]

    def _slot(self, L, i):
        return self.table[L][i // self.bs] * self.bs + i % self.bs

    def append(self, L, k, v, pos):
        need = self.count[L] + k.shape[0]
        while len(self.table[L]) * self.bs < need:
            self.table[L].append(self.pool.allocate())
        for i in range(k.shape[0]):
            s = self._slot(L, self.count[L])
            self.k_store[L][s] = k[i]
            self.v_store[L][s] = v[i]
            self.pos[L].append(int(pos[i]))
            self.count[L] += 1

    def read(self, L):
        n = self.count[L]
        slots = np.asarray([self._slot(L, i) for i in range(n)], np.int64)
        return self.k_store[L][slots], self.v_store[L][slots], np.asarray(self.pos[L], np.int64)

    def note_attention(self, L, probs):
        return None

    def truncate(self, n_pos):
        for L in range(self.n_layers):
            keep = sum(1 for p in self.pos[L] if p < n_pos)
            if keep == self.count[L]:
                continue
            self.pos[L] = self.pos[L][:keep]
            self.count[L] = keep
            need_blocks = -(-keep // self.bs)
            while len(self.table[L]) > need_blocks:
                self.pool.free(self.table[L].pop())

    @property
    def length(self):
        return self.count[0]
