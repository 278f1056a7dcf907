"""The reference crate's own unit tests, restated, run against BOTH the oracle
(CPU restatement) and the product host library (librmlx_kv.so).

Each test cites the Rust test it restates (crates/rmlx-serve-cache/src).
Passing on the oracle pins the oracle to the reference's known answers;
passing on the product shows the drop-in keeps them.
"""
import pytest

import oracle as orc
import rmlx_kv

IMPLS = {
    "oracle": (orc.PagedCacheManager, orc.PrefixCacheManager, orc.MemoryAwarePrefixCache),
    "product": (rmlx_kv.PagedCacheManager, rmlx_kv.PrefixCacheManager, rmlx_kv.MemoryAwarePrefixCache),
}


@pytest.fixture(params=["oracle", "product"])
def impl(request):
    return IMPLS[request.param]


def _tokens(mgr, b):
    blk = mgr.get_block(b)
    return blk[2] if isinstance(blk, tuple) else blk.tokens


def _filled(mgr, b):
    blk = mgr.get_block(b)
    return blk[3] if isinstance(blk, tuple) else blk.num_filled


# ---- paged_cache.rs:304-463 ----------------------------------------------

def test_new_manager(impl):  # :309-315
    m = impl[0](16, 100)
    assert m.num_free_blocks() == 100
    assert m.num_allocated_blocks() == 0


def test_allocate_and_free(impl):  # :318-348
    m = impl[0](16, 4)
    b0 = m.allocate()
    assert m.ref_count(b0) == 1
    assert m.num_free_blocks() == 3
    b1, b2, b3 = m.allocate(), m.allocate(), m.allocate()
    assert m.num_free_blocks() == 0
    assert m.allocate() is None
    m.free(b1)
    assert m.num_free_blocks() == 1
    assert m.ref_count(b1) == 0
    b4 = m.allocate()
    assert b4 == b1  # reused the freed block (FIFO)
    for b in (b0, b2, b3, b4):
        m.free(b)
    assert m.num_free_blocks() == 4


def test_ref_counting(impl):  # :351-372
    m = impl[0](16, 4)
    b0 = m.allocate()
    assert m.ref_count(b0) == 1
    m.increment_ref(b0)
    assert m.ref_count(b0) == 2
    m.increment_ref(b0)
    assert m.ref_count(b0) == 3
    m.free(b0)
    assert m.ref_count(b0) == 2
    assert m.num_free_blocks() == 3
    m.free(b0)
    assert m.ref_count(b0) == 1
    m.free(b0)
    assert m.ref_count(b0) == 0
    assert m.num_free_blocks() == 4


def test_copy_on_write_shared(impl):  # :375-396
    m = impl[0](16, 4)
    b0 = m.allocate()
    m.append_tokens(b0, [1, 2, 3])
    m.increment_ref(b0)
    assert m.ref_count(b0) == 2
    new_id = m.copy_on_write(b0)
    assert new_id is not None and new_id != b0
    assert m.ref_count(b0) == 1
    assert m.ref_count(new_id) == 1
    assert _tokens(m, new_id) == [1, 2, 3]
    assert _filled(m, new_id) == 3


def test_copy_on_write_unshared(impl):  # :399-405
    m = impl[0](16, 4)
    b0 = m.allocate()
    assert m.copy_on_write(b0) is None


def test_hash_lookup(impl):  # :408-419
    m = impl[0](16, 4)
    b0 = m.allocate()
    m.register_hash(b0, 12345)
    assert m.lookup_hash(12345) == b0
    assert m.lookup_hash(99999) is None
    m.free(b0)
    assert m.lookup_hash(12345) is None


def test_append_tokens(impl):  # :422-437
    m = impl[0](4, 2)
    b0 = m.allocate()
    m.append_tokens(b0, [10, 20])
    assert _tokens(m, b0) == [10, 20]
    assert _filled(m, b0) == 2
    m.append_tokens(b0, [30, 40])
    assert _tokens(m, b0) == [10, 20, 30, 40]
    assert _filled(m, b0) == 4


def test_append_tokens_overflow(impl):  # :440-445 (should_panic "overflow")
    m = impl[0](2, 1)
    b0 = m.allocate()
    with pytest.raises(RuntimeError, match="overflow"):
        m.append_tokens(b0, [1, 2, 3])


def test_double_free_panics(impl):  # :448-454 (should_panic "double free")
    m = impl[0](16, 2)
    b0 = m.allocate()
    m.free(b0)
    with pytest.raises(RuntimeError, match="double free"):
        m.free(b0)


def test_get_block(impl):  # :457-462
    m = impl[0](16, 2)
    assert m.get_block(0) is not None
    assert m.get_block(1) is not None
    assert m.get_block(2) is None


# ---- prefix_cache.rs:294-440 ---------------------------------------------

def test_new_prefix_cache(impl):  # :299-305
    c = impl[1](100)
    assert c.num_blocks() == 0
    assert c.max_blocks() == 100
    assert not c.is_full()
    assert c.hit_rate() == 0.0


def test_insert_and_lookup(impl):  # :308-331
    c = impl[1](100)
    c.insert([10, 20, 30, 40], [0, 1])
    assert c.lookup([10, 20, 30, 40]) == [0, 1]
    assert c.lookup([10, 20]) == [0]
    assert c.lookup([10, 20, 30]) == [0]
    assert c.lookup([99, 88]) == []


def test_single_block_insert(impl):  # :334-348
    c = impl[1](100)
    c.insert([1, 2, 3], [42])
    assert c.lookup([1, 2, 3]) == [42]
    assert c.lookup([1, 2]) == []


def test_overlapping_prefixes(impl):  # :351-366
    c = impl[1](100)
    c.insert([1, 2, 3], [10])
    c.insert([1, 2, 3, 4, 5, 6], [10, 20])
    assert c.lookup([1, 2, 3, 4, 5, 6]) == [10, 20]
    assert c.lookup([1, 2, 3]) == [10]


def test_evict_lru(impl):  # :369-387
    c = impl[1](2)
    c.insert([1, 2], [10])
    c.insert([3, 4], [20])
    assert c.num_blocks() == 2
    c.lookup([3, 4])
    assert c.evict_lru() == 10
    assert c.num_blocks() == 1
    assert c.lookup([3, 4]) == [20]


def test_evict_empty(impl):  # :390-393
    assert impl[1](10).evict_lru() is None


def test_hit_rate(impl):  # :396-409
    c = impl[1](100)
    c.insert([1, 2, 3], [10])
    c.lookup([1, 2, 3])
    assert c.hit_rate() > 0.0
    assert c.hit_rate() == pytest.approx(1 / 3)  # 1 block over 3 tokens (:401-403)
    c.lookup([99, 88, 77])
    assert c.hit_rate() == pytest.approx(1 / 6)  # (:408)


def test_insert_empty(impl):  # :412-419
    c = impl[1](100)
    c.insert([], [])
    assert c.num_blocks() == 0
    c.insert([1, 2], [])
    assert c.num_blocks() == 0


def test_branching_trie(impl):  # :422-439
    c = impl[1](100)
    c.insert([1, 2, 3, 4], [10, 11])
    c.insert([1, 2, 5, 6], [10, 12])
    assert c.lookup([1, 2, 3, 4]) == [10, 11]
    assert c.lookup([1, 2, 5, 6]) == [10, 12]
    assert c.lookup([1, 2]) == [10]


# ---- memory.rs:201-268 ---------------------------------------------------

def test_new_memory_aware_cache(impl):  # :206-211
    c = impl[2](100, 512)
    assert c.memory_limit_bytes() == 512 * 1024 * 1024
    assert c.current_usage_bytes() == 0
    assert c.num_blocks() == 0


def test_mem_insert_and_lookup(impl):  # :214-221
    c = impl[2](100, 512)
    c.insert([1, 2, 3], [10])
    c.insert([1, 2, 3, 4, 5, 6], [10, 20])
    assert c.lookup([1, 2, 3, 4, 5, 6]) == [10, 20]


def test_memory_tracking(impl):  # :224-233
    c = impl[2](100, 1, 1024)
    c.insert([1, 2], [10])
    assert c.current_usage_bytes() == 1024
    c.insert([3, 4], [20])
    assert c.current_usage_bytes() == 2048


def test_eviction_on_memory_pressure(impl):  # :236-246 (asserts nothing in the reference)
    c = impl[2](100, 0, 512)
    assert c.should_evict()  # limit 0: usage >= limit (:100)
    c.insert([1, 2], [10])
    assert c.current_usage_bytes() == 512
    assert c.num_blocks() == 1


def test_manual_evict(impl):  # :249-257
    c = impl[2](100, 512, 4096)
    c.insert([1, 2], [10])
    c.insert([3, 4], [20])
    assert c.evict_lru() is not None
    assert c.current_usage_bytes() == 4096


def test_available_memory():  # :260-267 (non-macOS build returns usize::MAX)
    assert rmlx_kv.MemoryAwarePrefixCache.available_memory_mb() == 2 ** 64 - 1


# ---- rotating_cache.rs:285-367 (oracle only: it defines the row-copy
# semantics that the paged append/gather follow) --------------------------

def test_rotating_append_linear():  # :300-314
    c = orc.RotatingKVCache(1, 1, 2, 4, 0)
    c.append(0, [1.0, 2.0, 3.0, 4.0], [10.0, 20.0, 30.0, 40.0], 2)
    assert c.seq_len() == 2
    assert c.get_keys(0) == [[1.0, 2.0, 3.0, 4.0]]
    assert c.get_values(0) == [[10.0, 20.0, 30.0, 40.0]]


def test_rotating_append_with_rotation():  # :317-341
    c = orc.RotatingKVCache(1, 1, 1, 3, 1)
    for i in range(3):
        c.append(0, [float(i + 1)], [float(i + 1) * 10], 1)
    assert c.seq_len() == 3
    assert c.get_keys(0)[0] == [1.0, 2.0, 3.0]
    c.append(0, [4.0], [40.0], 1)
    assert c.seq_len() == 3
    assert c.get_keys(0)[0] == [1.0, 3.0, 4.0]


def test_rotating_trim():  # :344-360
    c = orc.RotatingKVCache(1, 1, 1, 8, 2)
    for i in range(6):
        c.append(0, [float(i + 1)], [float(i + 1)], 1)
    assert c.seq_len() == 6
    c.trim(2)
    assert c.seq_len() == 4
    assert c.get_keys(0)[0] == [1.0, 2.0, 5.0, 6.0]


def test_rotating_keep_equals_max_size_panics():  # :363-366
    with pytest.raises(RuntimeError):
        orc.RotatingKVCache(1, 1, 1, 5, 5)
