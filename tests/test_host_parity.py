"""Randomised op-sequence parity of the product's host-side metadata
(librmlx_kv.so) against the oracle: after every operation the results
and the observable state must agree, including the reference's quirks
(FIFO reuse, hash entries that survive append_tokens, LRU ties broken by
arena index, leaves evicted before internal nodes)."""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv


def _same_exc(fa, fb):
    ea = eb = None
    ra = rb = None
    try:
        ra = fa()
    except RuntimeError as e:
        ea = e
    try:
        rb = fb()
    except RuntimeError as e:
        eb = e
    assert (ea is None) == (eb is None), (ea, eb)
    return ra, rb


@pytest.mark.parametrize("seed", range(6))
def test_block_manager_random_ops(seed):
    rng = np.random.default_rng(seed)
    bs, n = 4, 24
    A, B = rmlx_kv.PagedCacheManager(bs, n), orc.PagedCacheManager(bs, n)
    hashes = [int(x) for x in rng.integers(0, 2 ** 64 - 1, size=8, dtype=np.uint64)]
    for _ in range(3000):
        op = rng.integers(0, 8)
        bid = int(rng.integers(-1, n + 1)) if rng.random() < 0.1 else int(rng.integers(0, n))
        if op == 0:
            assert A.allocate() == B.allocate()
        elif op == 1:
            _same_exc(lambda: A.free(bid), lambda: B.free(bid))
        elif op == 2:
            _same_exc(lambda: A.increment_ref(bid), lambda: B.increment_ref(bid))
        elif op == 3:
            ra, rb = _same_exc(lambda: A.copy_on_write(bid), lambda: B.copy_on_write(bid))
            assert ra == rb
        elif op == 4:
            h = hashes[int(rng.integers(0, len(hashes)))]
            _same_exc(lambda: A.register_hash(bid, h), lambda: B.register_hash(bid, h))
        elif op == 5:
            h = hashes[int(rng.integers(0, len(hashes)))]
            assert A.lookup_hash(h) == B.lookup_hash(h)
        elif op == 6:
            toks = rng.integers(0, 100, size=int(rng.integers(0, 3))).tolist()
            _same_exc(lambda: A.append_tokens(bid, toks), lambda: B.append_tokens(bid, toks))
        else:
            if 0 <= bid < n:
                assert A.ref_count(bid) == B.ref_count(bid)
        assert A.num_free_blocks() == B.num_free_blocks()
        assert A.num_allocated_blocks() == B.num_allocated_blocks()
    for b in range(n):
        blk, ref = A.get_block(b), B.get_block(b)
        assert (blk.ref_count, blk.hash, blk.tokens, blk.num_filled) == ref


def _seq(rng, vocab, lo, hi):
    return rng.integers(0, vocab, size=int(rng.integers(lo, hi + 1))).tolist()


@pytest.mark.parametrize("seed", range(6))
def test_prefix_cache_random_ops(seed):
    """Small vocabulary so that prefixes collide, branch and get pruned."""
    rng = np.random.default_rng(100 + seed)
    A, B = rmlx_kv.PrefixCacheManager(64), orc.PrefixCacheManager(64)
    seen = []
    next_id = 0
    for _ in range(1500):
        r = rng.random()
        if r < 0.45:
            toks = _seq(rng, 4, 1, 12) if rng.random() < 0.7 or not seen else list(seen[int(rng.integers(len(seen)))])
            nb = int(rng.integers(0, 4))
            ids = list(range(next_id, next_id + nb))
            next_id += nb
            A.insert(toks, ids)
            B.insert(toks, ids)
            seen.append(toks)
        elif r < 0.8:
            toks = _seq(rng, 4, 0, 12) if rng.random() < 0.5 or not seen else seen[int(rng.integers(len(seen)))]
            assert A.lookup(toks) == B.lookup(toks)
        else:
            assert A.evict_lru() == B.evict_lru()
        assert A.num_blocks() == B.num_blocks()
        assert A.num_nodes() == B.num_nodes()
        assert A.is_full() == B.is_full()
    assert A.hit_rate() == B.hit_rate()
    order_a, order_b = [], []
    while True:
        a, b = A.evict_lru(), B.evict_lru()
        order_a.append(a)
        order_b.append(b)
        if a is None or b is None:
            break
    assert order_a == order_b


def test_prefix_cache_block_aligned_workload():
    """Shared 16-token-block prefixes (the prefix-caching config, scaled down):
    the whole eviction sequence must match."""
    rng = np.random.default_rng(0x5EED + 4)
    A, B = rmlx_kv.PrefixCacheManager(10 ** 6), orc.PrefixCacheManager(10 ** 6)
    prefixes = [rng.integers(0, 128256, size=128).tolist() for _ in range(4)]
    nid = 0
    for i in range(120):
        if rng.random() < 0.6:
            toks = prefixes[int(rng.integers(4))] + rng.integers(0, 128256, size=int(rng.integers(16, 64))).tolist()
        else:
            toks = rng.integers(0, 128256, size=int(rng.integers(32, 160))).tolist()
        toks = toks[:len(toks) // 16 * 16]
        hit_a, hit_b = A.lookup(toks), B.lookup(toks)
        assert hit_a == hit_b
        nb = len(toks) // 16
        ids = hit_a + list(range(nid, nid + nb - len(hit_a)))
        nid += nb - len(hit_a)
        A.insert(toks, ids)
        B.insert(toks, ids)
        if i % 7 == 0:
            for _ in range(5):
                assert A.evict_lru() == B.evict_lru()
    assert A.num_nodes() == B.num_nodes()
    ea, eb = [], []
    while A.num_blocks():
        ea.append(A.evict_lru())
        eb.append(B.evict_lru())
    assert ea == eb and B.num_blocks() == 0


@pytest.mark.parametrize("seed", range(3))
def test_memory_aware_random_ops(seed):
    rng = np.random.default_rng(200 + seed)
    A = rmlx_kv.MemoryAwarePrefixCache(40, 1, 4096 * 8)
    B = orc.MemoryAwarePrefixCache(40, 1, 4096 * 8)
    nid = 0
    for _ in range(600):
        r = rng.random()
        if r < 0.5:
            toks = _seq(rng, 6, 1, 10)
            nb = int(rng.integers(0, 3))
            ids = list(range(nid, nid + nb))
            nid += nb
            A.insert(toks, ids)
            B.insert(toks, ids)
        elif r < 0.85:
            toks = _seq(rng, 6, 0, 10)
            assert A.lookup(toks) == B.lookup(toks)
        else:
            assert A.evict_lru() == B.evict_lru()
        assert A.current_usage_bytes() == B.current_usage_bytes()
        assert A.num_blocks() == B.num_blocks()
        assert A.should_evict() == B.should_evict()
    assert A.drain_evicted() == B.evicted()
