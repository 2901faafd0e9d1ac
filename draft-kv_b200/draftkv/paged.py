"""Paged authoritative KV cache on the device, with the reference's rollback.

Same allocator semantics as the reference's draftkv/paged.py:29-181: a fixed
pool of blocks handed out and returned whole (LIFO free list), one block
table per layer, truncation frees whole trailing blocks and keeps the
partially filled tail, exhaustion raises BlockPoolExhausted, a double free
raises RuntimeError.  The allocator (block tables) stays on the host; the
K/V bytes live in one device pool [n_blocks][n_kv][block_size][d] per K and
V, addressed by the device page table [batch][n_layers][max_pages] that the
kernels read.

The device cache can hold several sequences (batch); the reference API
(append / read / truncate / length ...) addresses sequence 0.  Positions are
stored implicitly: entry i of a layer is position i (the reference only ever
appends consecutive positions to its authoritative cache).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import _lib

try:
    import torch
except ImportError:  # pragma: no cover - torch is a hard dependency of the device path
    torch = None


class BlockPoolExhausted(RuntimeError):
    """Raised instead of silently corrupting state when the pool runs dry."""


@dataclass
class BlockPool:
    """Fixed pool of KV blocks, handed out and returned by whole blocks
    (paged.py:33-74)."""

    n_blocks: int
    block_size: int
    _free: list = field(default_factory=list)
    _allocated: set = field(default_factory=set)

    def __post_init__(self) -> None:
        self._free = list(range(self.n_blocks))
        self._allocated = set()

    def allocate(self) -> int:
        if not self._free:
            raise BlockPoolExhausted(f"all {self.n_blocks} blocks of size {self.block_size} are in use")
        b = self._free.pop()
        self._allocated.add(b)
        return b

    def allocate_many(self, n: int) -> list:
        """n blocks in the order n calls of allocate() return them (the free
        list's last-in first-out order), in one slice."""
        if n > len(self._free):
            raise BlockPoolExhausted(f"all {self.n_blocks} blocks of size {self.block_size} are in use")
        if n <= 0:
            return []
        taken = self._free[-n:][::-1]
        del self._free[-n:]
        self._allocated.update(taken)
        return taken

    def free(self, block: int) -> None:
        if block not in self._allocated:
            raise RuntimeError(f"double free of block {block}")
        self._allocated.discard(block)
        self._free.append(block)

    @property
    def n_free(self) -> int:
        return len(self._free)

    @property
    def n_used(self) -> int:
        return len(self._allocated)

    def check_invariants(self) -> None:
        assert len(set(self._free)) == len(self._free), "duplicate in free list"
        assert not (set(self._free) & self._allocated), "block both free and allocated"
        assert len(self._free) + len(self._allocated) == self.n_blocks, "blocks leaked"


def plan_blocks_needed(ctx: int, n_layers: int, block_size: int) -> int:
    """Blocks a context of `ctx` tokens occupies across all layers (paged.py:179-181)."""
    return n_layers * (-(-ctx // block_size))


def dtype_code(dtype) -> int:
    """DKV_F32 / DKV_BF16 from a numpy / torch dtype or a name."""
    if dtype is None:
        return _lib.F32
    if isinstance(dtype, int) and dtype in (_lib.F32, _lib.BF16):
        return dtype
    if isinstance(dtype, str):
        return {"f32": _lib.F32, "float32": _lib.F32, "bf16": _lib.BF16, "bfloat16": _lib.BF16}[dtype]
    if torch is not None and dtype == torch.bfloat16:
        return _lib.BF16
    if torch is not None and dtype == torch.float32:
        return _lib.F32
    if np.dtype(dtype) == np.float32 or np.dtype(dtype) == np.float64:
        return _lib.F32
    raise ValueError(f"unsupported cache dtype {dtype!r}")


def torch_dtype(code: int):
    return torch.float32 if code == _lib.F32 else torch.bfloat16


class PagedKVCache:
    """The authoritative cache, stored in device blocks behind the cache
    interface (paged.py:76-177)."""

    def __init__(self, n_layers: int, n_heads: int, d_head: int, block_size: int = 16,
                 n_blocks: int = 512, dtype=np.float32, batch: int = 1,
                 max_blocks_per_seq: int | None = None, device: str = "cuda") -> None:
        self.n_layers = n_layers
        self.n_heads = n_heads          # KV heads (the cache holds KV heads)
        self.d_head = d_head
        self.block_size = block_size
        self.batch = batch
        self.dtype = dtype_code(dtype)
        self.pool = BlockPool(n_blocks, block_size)
        self.max_pages = max_blocks_per_seq or n_blocks
        self.device = device
        self._alloc_device(n_blocks)
        self.block_tables = [[[] for _ in range(n_layers)] for _ in range(batch)]
        self.counts = [[0] * n_layers for _ in range(batch)]

    # ------------------------------------------------------------ device
    def _alloc_device(self, n_blocks: int) -> None:
        _lib.load()
        td = torch_dtype(self.dtype)
        shape = (n_blocks, self.n_heads, self.block_size, self.d_head)
        self.k_pool = torch.zeros(shape, dtype=td, device=self.device)
        self.v_pool = torch.zeros(shape, dtype=td, device=self.device)
        self.table_host = torch.zeros((self.batch, self.n_layers, self.max_pages), dtype=torch.int32,
                                      pin_memory=True)
        self.table_dev = torch.zeros((self.batch, self.n_layers, self.max_pages), dtype=torch.int32,
                                     device=self.device)
        self._dirty = False
        self._struct = _lib.FullCacheS(self.k_pool.data_ptr(), self.v_pool.data_ptr(),
                                       self.table_dev.data_ptr(), n_blocks, self.block_size,
                                       self.max_pages, self.dtype)

    def struct(self) -> "_lib.FullCacheS":
        self.sync_table()
        return self._struct

    @property
    def host_resident(self) -> bool:
        return not self.k_pool.is_cuda

    def offload_to_host(self) -> None:
        """Moves the K/V pools to pinned host memory (configuration 5: a
        long context whose full cache is streamed from the host during verify,
        while the drafter cache stays in HBM).  The kernels read and write the
        pools in place through their unified addresses over the host link;
        page tables stay on the device.  Call between rounds."""
        if self.host_resident:
            return
        import torch
        torch.cuda.current_stream().synchronize()
        hk = torch.empty(self.k_pool.shape, dtype=self.k_pool.dtype, pin_memory=True)
        hk.copy_(self.k_pool)
        self.k_pool = hk
        hv = torch.empty(self.v_pool.shape, dtype=self.v_pool.dtype, pin_memory=True)
        hv.copy_(self.v_pool)
        self.v_pool = hv
        self._struct.k_pool = self.k_pool.data_ptr()
        self._struct.v_pool = self.v_pool.data_ptr()
        torch.cuda.empty_cache()

    def dims(self, batch: int | None = None) -> "_lib.DimsS":
        return _lib.DimsS(self.n_layers, self.n_heads, self.d_head, batch or self.batch)

    def sync_table(self) -> None:
        if self._dirty:
            self.table_dev.copy_(self.table_host)
            self._dirty = False

    @property
    def capacity_tokens(self) -> int:
        return self.max_pages * self.block_size

    # ------------------------------------------------- allocator (host)
    def ensure(self, b: int, n_tokens: int) -> None:
        """Blocks for positions [0, n_tokens) of sequence b in every layer."""
        need = -(-n_tokens // self.block_size)
        if need > self.max_pages:
            raise BlockPoolExhausted(f"sequence needs {need} blocks > max_blocks_per_seq {self.max_pages}")
        for L in range(self.n_layers):
            tbl = self.block_tables[b][L]
            if len(tbl) >= need:
                continue
            i0 = len(tbl)
            new = self.pool.allocate_many(need - i0)
            tbl.extend(new)
            row = self.table_host[b, L, i0:need]
            arr = torch.tensor(new, dtype=row.dtype)
            if not torch.equal(row, arr):
                row.copy_(arr)
                self._dirty = True

    def set_length(self, b: int, n: int) -> None:
        for L in range(self.n_layers):
            self.counts[b][L] = n

    def truncate_seq(self, b: int, n_pos: int) -> None:
        """paged.py:144-162 for one sequence: keep the prefix, free whole blocks."""
        for L in range(self.n_layers):
            keep = min(self.counts[b][L], n_pos)
            if keep == self.counts[b][L]:
                continue
            self.counts[b][L] = keep
            need = -(-keep // self.block_size)
            tbl = self.block_tables[b][L]
            while len(tbl) > need:
                self.pool.free(tbl.pop())

    def release_seq(self, b: int) -> None:
        self.truncate_seq(b, 0)

    # ---------------------------------------------------- cache protocol
    def append(self, layer: int, k, v, pos) -> None:
        k = np.asarray(k, np.float32)
        v = np.asarray(v, np.float32)
        pos = np.asarray(pos).reshape(-1)
        n = k.shape[0]
        start = self.counts[0][layer]
        if n == 0:
            return
        if not np.array_equal(pos, np.arange(start, start + n)):
            raise ValueError("the device cache stores consecutive positions starting at its length")
        need = -(-(start + n) // self.block_size)
        tbl = self.block_tables[0][layer]
        while len(tbl) < need:
            blk = self.pool.allocate()
            self.table_host[0, layer, len(tbl)] = blk
            tbl.append(blk)
            self._dirty = True
        src = np.stack([k, v], axis=2)                              # [n][h][2][d]
        t = torch.from_numpy(np.ascontiguousarray(src)).to(self.device, torch_dtype(self.dtype))
        p0 = torch.tensor([start], dtype=torch.int32, device=self.device)
        _lib.call("dkv_full_write", self.struct(), self.dims(1), layer, t.data_ptr(), n, p0.data_ptr(),
                  None, _lib.stream_ptr())
        self.counts[0][layer] = start + n

    def read(self, layer: int, b: int = 0):
        n = self.counts[b][layer]
        if n == 0:
            return (np.zeros((0, self.n_heads, self.d_head), np.float32),
                    np.zeros((0, self.n_heads, self.d_head), np.float32), np.zeros((0,), np.int64))
        out = torch.empty((n, self.n_heads, 2, self.d_head), dtype=torch_dtype(self.dtype), device=self.device)
        _lib.call("dkv_full_read", self.struct(), self.dims(), b, layer, n, out.data_ptr(), _lib.stream_ptr())
        o = out.float().cpu().numpy()
        return o[:, :, 0, :], o[:, :, 1, :], np.arange(n, dtype=np.int64)

    def note_attention(self, layer: int, probs) -> None:  # the full cache keeps no scores
        return None

    def truncate(self, n_pos: int) -> None:
        for b in range(self.batch):
            self.truncate_seq(b, n_pos)

    @property
    def length(self) -> int:
        return self.counts[0][0]

    @property
    def blocks_in_use(self) -> int:
        return self.pool.n_used

    def fragmentation(self) -> float:
        cap = self.pool.n_used * self.block_size
        live = sum(sum(c) for c in self.counts)
        return 0.0 if cap == 0 else 1.0 - live / cap

    @property
    def pos(self):
        return [[list(range(c)) for c in seq] for seq in self.counts][0]
