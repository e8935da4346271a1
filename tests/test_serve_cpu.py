"""Host-side serving logic: block manager, prefix cache, eviction."""
import pytest

from lora_kernel_b200.serve.kv_cache import BlockManager, block_hashes


def test_hash_chain_depends_on_prefix():
    a = block_hashes(list(range(64)), 16)
    b = block_hashes([99] + list(range(1, 64)), 16)
    assert len(a) == 4 and all(x != y for x, y in zip(a, b))


def test_allocate_share_release_evict():
    bm = BlockManager(num_blocks=10, block_size=4)
    p = list(range(10))                      # 2 full blocks + tail
    t1, c1 = bm.allocate(p)
    assert c1 == 0 and len(t1) == 3
    bm.register_full_blocks(p, t1, len(p))
    t2, c2 = bm.allocate(p[:8] + [50, 51, 52])
    assert c2 == 8 and t2[:2] == t1[:2] and bm.ref[t1[0]] == 2
    assert bm.stats.hits == 2
    bm.free_seq(t1)
    bm.free_seq(t2)
    assert bm.num_free() == 10 and len(bm.evictable) == 2
    # cached blocks survive until the allocator needs them
    t3, c3 = bm.allocate(p)
    assert c3 == 8
    bm.free_seq(t3)
    big, _ = bm.allocate(list(range(100, 140)))  # 10 blocks: evicts the cached ones
    assert bm.stats.evictions == 2 and len(bm.block_of) == 0
    with pytest.raises(MemoryError):
        bm.allocate([1])
    bm.free_seq(big)


def test_append_slot_grows_table():
    bm = BlockManager(num_blocks=4, block_size=4)
    t, _ = bm.allocate([1, 2, 3, 4])
    assert len(t) == 1
    s = bm.append_slot(t, 4)
    assert len(t) == 2 and s == t[1] * 4
    assert bm.slots_for(t, 3, 5) == [t[0] * 4 + 3, t[1] * 4]


def test_full_prompt_hit_keeps_last_token_uncached():
    bm = BlockManager(num_blocks=8, block_size=4)
    p = list(range(8))
    t, _ = bm.allocate(p)
    bm.register_full_blocks(p, t, 8)
    t2, cached = bm.allocate(p)
    assert cached == 4  # the block holding the last token is recomputed
