"""Host-side page allocation of the paged full cache (no GPU): `ensure`
takes a layer's missing pages in one slice of the block pool's free list and
must hand out exactly the blocks, in exactly the order, that allocating one
page at a time does (the last-in first-out order of draftkv/paged.py:33-74,
which the golden paged traces pin)."""
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "draft-kv_b200"))

from draftkv.paged import BlockPool, PagedKVCache  # noqa: E402


def _host_cache(n_layers, batch, n_blocks, block_size=16, max_pages=64):
    # the allocator state of a PagedKVCache without its device pools
    c = object.__new__(PagedKVCache)
    c.n_layers, c.batch, c.block_size, c.max_pages = n_layers, batch, block_size, max_pages
    c.pool = BlockPool(n_blocks, block_size)
    c.block_tables = [[[] for _ in range(n_layers)] for _ in range(batch)]
    c.table_host = torch.zeros((batch, n_layers, max_pages), dtype=torch.int32)
    c._dirty = False
    return c


def _ensure_one_at_a_time(c, b, n_tokens):
    need = -(-n_tokens // c.block_size)
    for L in range(c.n_layers):
        tbl = c.block_tables[b][L]
        while len(tbl) < need:
            blk = c.pool.allocate()
            tbl.append(blk)
            c.table_host[b, L, len(tbl) - 1] = blk


def test_allocate_many_matches_allocate():
    p1, p2 = BlockPool(100, 16), BlockPool(100, 16)
    first = p2.allocate_many(7)
    assert [p1.allocate() for _ in range(7)] == first == list(range(99, 92, -1))
    p1.free(97), p2.free(97)
    p1.free(95), p2.free(95)
    assert [p1.allocate() for _ in range(4)] == p2.allocate_many(4)
    assert p2.allocate_many(0) == []
    p2.check_invariants()


def test_ensure_hands_out_the_one_at_a_time_blocks():
    a, b = _host_cache(3, 2, 400), _host_cache(3, 2, 400)
    steps = [(0, 40), (1, 17), (0, 41), (1, 200), (0, 300), (1, 16)]
    for s, n in steps:
        a.ensure(s, n)
        _ensure_one_at_a_time(b, s, n)
        assert a.block_tables == b.block_tables
        assert torch.equal(a.table_host, b.table_host)
    # a freed block comes back first, as allocate() would hand it out
    blk = a.block_tables[1][2].pop()
    a.pool.free(blk)
    b.pool.free(b.block_tables[1][2].pop())
    a.ensure(1, 400)
    _ensure_one_at_a_time(b, 1, 400)
    assert a.block_tables == b.block_tables
    assert torch.equal(a.table_host, b.table_host)
    assert a._dirty
    a.pool.check_invariants()
