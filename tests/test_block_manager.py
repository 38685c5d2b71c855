"""Paged block manager semantics (reference: src/memory/kv_cache_manager.cpp)."""
import pytest


def test_null_block_and_capacity(host):
    bm = host.BlockManager(10, 16, True)
    assert bm.num_free_blocks == 9            # block 0 is the null block
    assert bm.allocate(1, 16 * 9)
    assert 0 not in bm.blocks_of(1)
    assert not bm.allocate(2, 1)
    bm.free(1)
    assert bm.num_free_blocks == 9


def test_allocate_incremental_and_failure_is_atomic(host):
    bm = host.BlockManager(6, 16, True)
    assert bm.allocate(1, 10) and len(bm.blocks_of(1)) == 1
    assert bm.allocate(1, 17) and len(bm.blocks_of(1)) == 2
    assert bm.allocate(1, 32) and len(bm.blocks_of(1)) == 2
    before = bm.num_free_blocks
    assert not bm.allocate(2, 16 * 10)
    assert bm.num_free_blocks == before and bm.blocks_of(2) == []


def test_lru_free_order_tail_first(host):
    bm = host.BlockManager(8, 4, True)
    bm.allocate(1, 12)                       # blocks 1,2,3
    bm.allocate(2, 4)                        # block 4
    b1 = bm.blocks_of(1)
    bm.free(1)                               # appended tail-first: 3,2,1 after 5,6,7
    bm.allocate(3, 4 * 6)
    got = bm.blocks_of(3)
    assert got[:3] == [5, 6, 7] and got[3:] == list(reversed(b1))


def test_prefix_cache_hit_and_eviction(host):
    bm = host.BlockManager(6, 4, True)
    toks = list(range(12))
    hashes = host.BlockManager.block_hashes(toks, 4)
    assert len(hashes) == 3
    bm.allocate(1, 12)
    bm.cache_full_blocks(1, hashes, 3)
    blocks = bm.blocks_of(1)
    bm.free(1)
    hits = bm.find_longest_prefix_hit(hashes, 2)
    assert hits == blocks[:2]
    assert bm.allocate(2, 12, hits)           # shares the cached blocks
    assert bm.blocks_of(2)[:2] == blocks[:2]
    bm.free(2)
    # exhaust the pool: cached blocks get evicted (hash dropped)
    assert bm.allocate(3, 4 * 5)
    assert bm.find_longest_prefix_hit(hashes, 3) == []


def test_chained_hash_depends_on_prefix(host):
    a = host.BlockManager.block_hashes([1, 2, 3, 4, 5, 6, 7, 8], 4)
    b = host.BlockManager.block_hashes([9, 2, 3, 4, 5, 6, 7, 8], 4)
    assert a[0] != b[0] and a[1] != b[1]
    c = host.BlockManager.block_hashes([1, 2, 3, 4, 5, 6, 7, 9], 4)
    assert a[0] == c[0] and a[1] != c[1]


def test_refcount_shared_blocks(host):
    bm = host.BlockManager(8, 4, True)
    h = host.BlockManager.block_hashes(list(range(8)), 4)
    bm.allocate(1, 8)
    bm.cache_full_blocks(1, h, 2)
    hits = bm.find_longest_prefix_hit(h, 2)
    bm.allocate(2, 8, hits)
    free_before = bm.num_free_blocks
    bm.free(1)
    assert bm.num_free_blocks == free_before      # still referenced by request 2
    bm.free(2)
    assert bm.num_free_blocks == free_before + 2


def test_trim(host):
    bm = host.BlockManager(8, 4, True)
    bm.allocate(1, 16)
    bm.trim(1, 5)
    assert len(bm.blocks_of(1)) == 2
    with pytest.raises(RuntimeError):
        bm.trim(1, -1)
