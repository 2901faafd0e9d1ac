"""Device KV caches behind the reference's cache interface.

quantize            -- group quantization, bit-identical to the reference's
                       draftkv/compress.py:21-46 (device kernel dkv_quantize)
FullKVCache         -- exact authoritative cache (compress.py:49-92), here a
                       paged device cache that sizes itself on first use
CompressedKVCache   -- the drafter's quantized, eviction-pruned mirror
                       (compress.py:95-241): device slot arrays per
                       (sequence, layer); append / evict / truncate / resync /
                       rebuild run as fused kernels; attention mass is
                       accumulated by the draft-attention kernel itself, so
                       note_attention is a no-op here

Device layouts are documented in include/draftkv_b200.h.
"""

from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import _lib
from .config import CompressionConfig, LayerPlan
from .paged import PagedKVCache, dtype_code, torch_dtype

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


def quantize(x, bits: int, group: int = 64):
    """Round-trip `x` through a `bits`-wide affine grid per group of `group`
    channels on the device; returns the dequantized fp32 array (numpy in,
    numpy out; torch CUDA tensor in, tensor out).  Bit-identical to the
    reference's quantize (compress.py:21-46)."""
    if group != 64:
        raise ValueError("the device quantizer uses groups of 64")
    as_numpy = not (torch is not None and isinstance(x, torch.Tensor))
    t = torch.as_tensor(np.asarray(x, np.float32) if as_numpy else x, dtype=torch.float32)
    shape = t.shape
    t = t.reshape(-1, shape[-1]).contiguous().to("cuda")
    out = torch.empty_like(t)
    _lib.call("dkv_quantize", t.data_ptr(), t.shape[0], t.shape[1], int(bits), None, None, None,
              out.data_ptr(), _lib.stream_ptr())
    out = out.reshape(shape)
    return out.cpu().numpy() if as_numpy else out


def quantize_codes(x, bits: int):
    """(codes uint8 [rows, ceil(d/64)*64], scale f32, lo f32, deq f32) -- the
    locals of compress.py:38-43 made visible, computed on the device."""
    t = torch.as_tensor(np.asarray(x, np.float32)).reshape(-1, np.shape(x)[-1]).contiguous().to("cuda")
    rows, d = t.shape
    ng = -(-d // 64)
    codes = torch.empty((rows, ng * 64), dtype=torch.uint8, device="cuda")
    scale = torch.empty((rows, ng), dtype=torch.float32, device="cuda")
    lo = torch.empty((rows, ng), dtype=torch.float32, device="cuda")
    deq = torch.empty_like(t)
    _lib.call("dkv_quantize", t.data_ptr(), rows, d, int(bits), codes.data_ptr(), scale.data_ptr(),
              lo.data_ptr(), deq.data_ptr(), _lib.stream_ptr())
    return (codes.cpu().numpy(), scale.cpu().numpy(), lo.cpu().numpy(),
            deq.cpu().numpy().reshape(np.shape(x)))


class FullKVCache(PagedKVCache):
    """Exact cache (compress.py:49-92).  Shape and dtype are learned from the
    first model that writes into it; capacity grows by whole pools."""

    def __init__(self, n_layers: int, n_kv: int | None = None, d_head: int | None = None,
                 dtype=None, capacity: int = 2048, block_size: int = 16, batch: int = 1) -> None:
        self.n_layers = n_layers
        self._capacity = capacity
        self._bs = block_size
        self._batch = batch
        self._ready = False
        if n_kv is not None and d_head is not None:
            self.materialize(n_kv, d_head, dtype)

    def materialize(self, n_kv: int, d_head: int, dtype) -> None:
        if self._ready:
            return
        pages = -(-self._capacity // self._bs)
        super().__init__(self.n_layers, n_kv, d_head, block_size=self._bs,
                         n_blocks=pages * self.n_layers * self._batch, dtype=dtype,
                         batch=self._batch, max_blocks_per_seq=pages)
        self._ready = True

    def grow(self, need_tokens: int) -> None:
        """Reallocates the pool for at least `need_tokens` per sequence."""
        if need_tokens <= self.capacity_tokens:
            return
        cap = max(need_tokens, 2 * self.capacity_tokens)
        pages = -(-cap // self.block_size)
        old_k, old_v, old_tables, old_counts = self.k_pool, self.v_pool, self.block_tables, self.counts
        old_pool = self.pool
        from .paged import BlockPool
        self.pool = BlockPool(pages * self.n_layers * self.batch, self.block_size)
        self.max_pages = pages
        self._alloc_device(self.pool.n_blocks)
        self.block_tables = [[[] for _ in range(self.n_layers)] for _ in range(self.batch)]
        self.counts = [[0] * self.n_layers for _ in range(self.batch)]
        # move live blocks
        for b in range(self.batch):
            for L in range(self.n_layers):
                for blk in old_tables[b][L]:
                    nb = self.pool.allocate()
                    self.table_host[b, L, len(self.block_tables[b][L])] = nb
                    self.block_tables[b][L].append(nb)
                    self.k_pool[nb].copy_(old_k[blk])
                    self.v_pool[nb].copy_(old_v[blk])
                self.counts[b][L] = old_counts[b][L]
        self._dirty = True
        del old_pool

    @property
    def length(self) -> int:
        return self.counts[0][0] if self._ready else 0

    def append(self, layer, k, v, pos):
        if not self._ready:
            self.materialize(k.shape[1], k.shape[2], np.float32)
        self.grow(self.counts[0][layer] + k.shape[0])
        super().append(layer, k, v, pos)

    def read(self, layer, b: int = 0):
        if not self._ready:
            return (np.zeros((0, 0, 0), np.float32), np.zeros((0, 0, 0), np.float32), np.zeros((0,), np.int64))
        return super().read(layer, b)

    def truncate(self, n_pos: int) -> None:
        if self._ready:
            super().truncate(n_pos)


def _layer_cfgs(cfg, n_layers: int) -> list[CompressionConfig]:
    if isinstance(cfg, LayerPlan):
        cfgs = list(cfg.cfgs)
    elif isinstance(cfg, CompressionConfig):
        cfgs = [cfg] * n_layers
    else:
        cfgs = list(cfg)
    if len(cfgs) != n_layers:
        raise ValueError(f"expected {n_layers} per-layer configs, got {len(cfgs)}")
    return cfgs


class CompressedKVCache:
    """The drafter's lossy view on the device (compress.py:95-241).

    Per (sequence, layer) a slot array of `cap` entries: packed K/V codes,
    fp16 (scale, lo) per 64-group, position (-1 = empty) and accumulated
    attention mass.  Eviction keeps the `sink` lowest and `recent` highest
    positions and drops the lowest accumulated mass first (ties: lowest
    position), down to max(round(keep * seen), sink + recent).
    """

    def __init__(self, n_layers: int, cfg, n_kv: int | None = None, d_head: int | None = None,
                 dtype=None, capacity: int = 1024, batch: int = 1, max_bits: int = 16) -> None:
        self.n_layers = n_layers
        self.cfgs = _layer_cfgs(cfg, n_layers)
        self.cfg = self.cfgs[0]
        self.batch = batch
        self._capacity = capacity
        self._max_bits = max_bits
        self._ready = False
        self._cfg_arrays()
        if n_kv is not None and d_head is not None:
            self.materialize(n_kv, d_head, dtype)

    # ---------------------------------------------------------- storage
    def _cfg_arrays(self) -> None:
        n = self.n_layers
        self._bits = (C.c_int32 * n)(*[c.bits for c in self.cfgs])
        self._keep = (C.c_double * n)(*[c.keep_frac for c in self.cfgs])
        self._sink = (C.c_int32 * n)(*[c.sink for c in self.cfgs])
        self._recent = (C.c_int32 * n)(*[c.recent for c in self.cfgs])
        if self._ready:
            self._refresh_struct()

    def materialize(self, n_kv: int, d_head: int, dtype) -> None:
        if self._ready:
            return
        _lib.load()
        if d_head % 64:
            raise ValueError(f"the device drafter cache needs head_dim % 64 == 0 (got {d_head})")
        self.n_kv, self.d_head = n_kv, d_head
        self.dtype = dtype_code(dtype)
        self._alloc(self._capacity)
        self._ready = True

    def _alloc(self, cap: int) -> None:
        B, L, H, d = self.batch, self.n_layers, self.n_kv, self.d_head
        elem = 4 if self.dtype == _lib.F32 else 2
        self.cb_max = d * elem if self._max_bits >= 16 else d * self._max_bits // 8
        if self.dtype == _lib.F32 and self.cb_max < d * 4:
            self.cb_max = max(self.cb_max, 0)
        cap = -(-cap // 16) * 16          # whole 16-slot tiles (the tensor-core kernel copies tiles)
        self.cap = cap
        dev = "cuda"
        self.k_codes = torch.zeros((B, L, H, cap, self.cb_max), dtype=torch.uint8, device=dev)
        self.v_codes = torch.zeros_like(self.k_codes)
        self.k_sl = torch.zeros((B, L, H, cap, d // 64, 2), dtype=torch.int16, device=dev)
        self.v_sl = torch.zeros_like(self.k_sl)
        self.pos_t = torch.full((B, L, cap), -1, dtype=torch.int32, device=dev)
        self.score_t = torch.zeros((B, L, cap), dtype=torch.float32, device=dev)
        self.mass_t = torch.zeros((B, L, H, cap), dtype=torch.float32, device=dev)
        self.meta_t = torch.zeros((B, L, 4), dtype=torch.int32, device=dev)
        self.seen_t = torch.zeros((B,), dtype=torch.int32, device=dev)
        self.tickets_t = torch.zeros((B, L, 64), dtype=torch.int32, device=dev)
        self._refresh_struct()

    def _refresh_struct(self) -> None:
        self._s = _lib.CompCacheS(
            self.k_codes.data_ptr(), self.v_codes.data_ptr(), self.k_sl.data_ptr(), self.v_sl.data_ptr(),
            self.pos_t.data_ptr(), self.score_t.data_ptr(), self.mass_t.data_ptr(), self.meta_t.data_ptr(),
            self.seen_t.data_ptr(), self.tickets_t.data_ptr(), self.cap, self.cb_max,
            C.cast(self._bits, C.c_void_p), C.cast(self._keep, C.c_void_p),
            C.cast(self._sink, C.c_void_p), C.cast(self._recent, C.c_void_p))

    def struct(self) -> "_lib.CompCacheS":
        return self._s

    def dims(self) -> "_lib.DimsS":
        return _lib.DimsS(self.n_layers, self.n_kv, self.d_head, self.batch)

    def _grow(self, need: int) -> None:
        if need <= self.cap:
            return
        old = (self.k_codes, self.v_codes, self.k_sl, self.v_sl, self.pos_t, self.score_t, self.meta_t,
               self.seen_t)
        oc = self.cap
        self._alloc(max(need, 2 * oc))
        self.k_codes[:, :, :, :oc] = old[0]
        self.v_codes[:, :, :, :oc] = old[1]
        self.k_sl[:, :, :, :oc] = old[2]
        self.v_sl[:, :, :, :oc] = old[3]
        self.pos_t[:, :, :oc] = old[4]
        self.score_t[:, :, :oc] = old[5]
        self.meta_t.copy_(old[6])
        self.seen_t.copy_(old[7])

    @property
    def max_bits(self) -> int:
        """Widest code the slot arrays were sized for (16: raw entries)."""
        return self._max_bits

    def set_cfgs(self, cfgs: Sequence[CompressionConfig]) -> None:
        self.cfgs = list(cfgs)
        self.cfg = self.cfgs[0]
        self._cfg_arrays()

    # ---------------------------------------------------- host mirrors
    @property
    def seen_positions(self) -> int:
        return int(self.seen_t[0].item()) if self._ready else 0

    def budget(self, layer: int = 0) -> int:
        c = self.cfgs[layer]
        return max(int(round(c.keep_frac * max(self.seen_positions, 1))), c.sink + c.recent)

    def _hwm_max(self) -> int:
        return int(self.meta_t[:, :, 0].max().item())

    def _kept_after_fill(self, n: int, seen: int, layers) -> int:
        """Entries a layer keeps after `n` rows are appended to it empty with
        zero scores (the rebuild path writes only those)."""
        most = 0
        for L in layers:
            c = self.cfgs[L]
            budget = max(int(round(c.keep_frac * max(seen, 1))), c.sink + c.recent)
            most = max(most, n if (n <= budget or c.recent <= 0) else budget)
        return most

    # ---------------------------------------------------- protocol
    def append(self, layer: int, k, v, pos) -> None:
        """Quantize rows into free slots with score 0, then evict once
        (compress.py:122-133)."""
        k = np.asarray(k, np.float32)
        v = np.asarray(v, np.float32)
        pos = np.asarray(pos).reshape(-1)
        if not self._ready:
            self.materialize(k.shape[1], k.shape[2], np.float32)
        n = k.shape[0]
        if n == 0:
            return
        if not np.array_equal(pos, np.arange(pos[0], pos[0] + n)):
            raise ValueError("appended positions must be consecutive")
        self._grow(self._hwm_max() + n + 1)
        src = torch.from_numpy(np.ascontiguousarray(np.stack([k, v], axis=2))).to("cuda", torch_dtype(self.dtype))
        p0 = torch.tensor([int(pos[0])], dtype=torch.int32, device="cuda")
        nr = torch.tensor([n], dtype=torch.int32, device="cuda")
        _lib.call("dkv_comp_append", self.struct(), None, self.dims(), layer, 1, src.data_ptr(), self.dtype, n,
                  p0.data_ptr(), nr.data_ptr(), None, 1 if layer == 0 else 0, _lib.stream_ptr())

    def code_rows(self, which: str, layer: int, b: int = 0):
        """Packed codes ("k" or "v") of one layer and sequence as a
        [n_kv][cap][bytes per vector] view: a layer's vectors are stored
        densely at the width of its current configuration inside each
        (sequence, layer, head) region of the allocation."""
        bits, d = self.cfgs[layer].bits, self.d_head
        kb = d * (4 if self.cb_max >= d * 4 else 2) if bits >= 16 else d * bits // 8
        t = getattr(self, which + "_codes")[b, layer]                # [n_kv][cap][cb_max]
        return t.reshape(t.shape[0], -1)[:, : self.cap * kb].reshape(t.shape[0], self.cap, kb)

    def read(self, layer: int, b: int = 0):
        """Dequantized (k, v, pos) of the live entries in position order."""
        if not self._ready:
            return (np.zeros((0, 0, 0), np.float32), np.zeros((0, 0, 0), np.float32), np.zeros((0,), np.int64))
        k, v, p, s = self._read_slots(layer, b)
        order = np.argsort(p[p >= 0], kind="stable")
        live = np.nonzero(p >= 0)[0][order]
        return k[live], v[live], p[live].astype(np.int64)

    def scores(self, layer: int, b: int = 0):
        """(positions, accumulated mass) of the live entries in position order."""
        k, v, p, s = self._read_slots(layer, b)
        live = np.nonzero(p >= 0)[0]
        live = live[np.argsort(p[live], kind="stable")]
        return p[live].astype(np.int64), s[live]

    def _read_slots(self, layer: int, b: int):
        n_max = self.cap
        kk = torch.empty((n_max, self.n_kv, self.d_head), dtype=torch.float32, device="cuda")
        vv = torch.empty_like(kk)
        pp = torch.empty((n_max,), dtype=torch.int32, device="cuda")
        ss = torch.empty((n_max,), dtype=torch.float32, device="cuda")
        n = C.c_int(0)
        _lib.call("dkv_comp_read", self.struct(), self.dims(), b, layer, n_max, kk.data_ptr(), vv.data_ptr(),
                  pp.data_ptr(), ss.data_ptr(), C.byref(n), _lib.stream_ptr())
        m = n.value
        return (kk[:m].cpu().numpy(), vv[:m].cpu().numpy(), pp[:m].cpu().numpy(), ss[:m].cpu().numpy())

    def note_attention(self, layer: int, probs, b: int = 0) -> None:
        """compress.py:144-151: add probs summed over (query, head) to the live
        entries in position order.  Draft forwards do not call this: the
        draft-attention kernel accumulates the same mass itself."""
        probs = np.asarray(probs)
        if probs.size == 0 or not self._ready:
            return
        mass = probs.sum(axis=(0, 1)).astype(np.float32)
        pos = self.pos_t[b, layer].cpu().numpy()
        live = np.nonzero(pos >= 0)[0]
        live = live[np.argsort(pos[live], kind="stable")]
        n = min(len(live), mass.shape[0])
        if n:
            idx = torch.from_numpy(live[:n].astype(np.int64)).to("cuda")
            self.score_t[b, layer].index_add_(0, idx, torch.from_numpy(mass[:n]).to("cuda"))

    def truncate(self, n_pos: int) -> None:
        """compress.py:181-188: drop entries at positions >= n_pos, clip seen."""
        if not self._ready:
            return
        B = self.batch
        zero = torch.zeros((B,), dtype=torch.int32, device="cuda")
        tr = torch.full((B,), int(n_pos), dtype=torch.int32, device="cuda")
        _lib.call("dkv_comp_append", self.struct(), None, self.dims(), 0, self.n_layers, None, self.dtype, 0,
                  zero.data_ptr(), zero.data_ptr(), tr.data_ptr(), 0, _lib.stream_ptr())

    def sync_from(self, full: PagedKVCache, start_pos: int) -> int:
        """compress.py:190-207: drop positions >= start_pos and re-append the
        true K/V rows from the full cache.  Returns rows rewritten."""
        n = full.length
        if not self._ready:
            self.materialize(full.n_heads, full.d_head, full.dtype)
        rows = max(0, n - start_pos)
        if start_pos == 0:
            # everything is rewritten: clear, then refill every layer with the
            # rows that survive eviction at zero scores
            self.seen_t.zero_()
            self._grow(self._kept_after_fill(n, n, range(self.n_layers)) + 1)
            ctx = torch.full((self.batch,), n, dtype=torch.int32, device="cuda")
            layers = (C.c_int32 * self.n_layers)(*range(self.n_layers))
            _lib.call("dkv_comp_rebuild", self.struct(), full.struct(), self.dims(), layers, self.n_layers,
                      ctx.data_ptr(), 1, _lib.stream_ptr())
            return rows * self.n_layers
        self._grow(self._hwm_max() + rows + 1)
        B = self.batch
        p0 = torch.full((B,), start_pos, dtype=torch.int32, device="cuda")
        nr = torch.full((B,), rows, dtype=torch.int32, device="cuda")
        _lib.call("dkv_comp_append", self.struct(), full.struct(), self.dims(), 0, self.n_layers, None,
                  full.dtype, max(rows, 1), p0.data_ptr(), nr.data_ptr(), p0.data_ptr(), 1, _lib.stream_ptr())
        return rows * self.n_layers

    def rebuild_layers(self, full: PagedKVCache, layers, cfgs=None) -> int:
        """compress.py:209-230: clear and requantize only the named layers."""
        layers = list(layers)
        if cfgs is not None:
            new = list(self.cfgs)
            for L in layers:
                new[L] = cfgs[L]
            self.set_cfgs(new)
        if not layers:
            return 0
        n = full.length
        if not self._ready:
            self.materialize(full.n_heads, full.d_head, full.dtype)
        seen = max(self.seen_positions, n) if 0 in layers else self.seen_positions
        self._grow(self._kept_after_fill(n, seen, layers) + 1)
        ctx = torch.full((self.batch,), n, dtype=torch.int32, device="cuda")
        arr = (C.c_int32 * len(layers))(*layers)
        _lib.call("dkv_comp_rebuild", self.struct(), full.struct(), self.dims(), arr, len(layers),
                  ctx.data_ptr(), 1, _lib.stream_ptr())
        return n * len(layers)

    @property
    def length(self) -> int:
        if not self._ready:
            return 0
        return int(self.meta_t[0, 0, 1].item())

    def nbytes(self, n_heads: int, d_head: int) -> float:
        """Bytes held, summed per layer (compress.py:236-241)."""
        counts = self.meta_t[0, :, 1].tolist() if self._ready else [0] * self.n_layers
        return sum(2.0 * counts[L] * n_heads * self.cfgs[L].bytes_per_entry(d_head)
                   for L in range(self.n_layers))
