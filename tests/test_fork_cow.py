"""Forked decode batches over the block manager (host logic, no GPU).

SequenceBlocks driven by this package's PagedCacheManager and by the
oracle's restatement of paged_cache.rs must hand out the same blocks, the
same copy-on-write pairs and the same slots on every step (block tables are
bit-exact), and every block's reference count must equal the number of
tables that hold it.
"""
from collections import Counter

import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from rmlx_kv.batch import PoolExhausted, SequenceBlocks


def _drive(mgr, lens, steps, nfork, bs, seed):
    rng = np.random.default_rng(seed)
    seqs = SequenceBlocks(mgr, bs, lens)
    out = []
    for _ in range(steps):
        idx = rng.permutation(len(lens))
        for p, c in zip(idx[:nfork], idx[nfork:2 * nfork]):
            seqs.fork(int(p), int(c))
        src, dst, slots = seqs.append_slots()
        out.append((src, dst, slots, seqs.block_table(), seqs.seq_lens()))
    return seqs, out


@pytest.mark.parametrize("bs", [16, 1, 7])
def test_fork_plans_match_oracle_manager(bs):
    rng = np.random.default_rng(40 + bs)
    lens = rng.integers(0, 90, size=24)
    nb = int(((lens + bs - 1) // bs).sum()) + 12 * (24 + 4) + 8
    a, pa = _drive(rmlx_kv.PagedCacheManager(bs, nb), lens, 12, 4, bs, 7)
    b, pb = _drive(orc.PagedCacheManager(bs, nb), lens, 12, 4, bs, 7)
    cows = 0
    for x, y in zip(pa, pb):
        for u, v in zip(x, y):
            np.testing.assert_array_equal(u, v)
        cows += len(x[0])
    assert cows > 0 or bs == 1  # shared partial tails were extended (bs 1: every block is full)
    held = Counter(blk for t in a.tables for blk in t)
    for blk in range(nb):
        assert a.mgr.ref_count(blk) == held.get(blk, 0) == b.mgr.ref_count(blk)
    assert a.mgr.num_free_blocks() == b.mgr.num_free_blocks() == nb - len(held)


def test_cow_only_when_tail_shared():
    m = rmlx_kv.PagedCacheManager(4, 16)
    s = SequenceBlocks(m, 4, [6, 0])
    s.fork(0, 1)  # child shares both blocks; the tail (2 of 4 filled) is shared
    shared_tail = s.tables[0][1]
    src, dst, slots = s.append_slots()
    # sequence 0 writes first and gets the private copy; sequence 1 is then
    # the tail's only holder and writes in place
    assert src.tolist() == [shared_tail] and dst.tolist() == [s.tables[0][1]]
    assert s.tables[1][1] == shared_tail and m.ref_count(shared_tail) == 1
    assert slots.tolist() == [s.tables[0][1] * 4 + 2, s.tables[1][1] * 4 + 2]
    assert s.tables[0][0] == s.tables[1][0] and m.ref_count(s.tables[0][0]) == 2
    src, dst, _ = s.append_slots()  # tails now private: no copy
    assert len(src) == 0 and len(dst) == 0


def test_fork_at_block_boundary_needs_no_copy():
    m = rmlx_kv.PagedCacheManager(4, 16)
    s = SequenceBlocks(m, 4, [8, 3])
    s.fork(0, 1)
    src, _, slots = s.append_slots()  # both start a fresh block
    assert len(src) == 0 and s.tables[0][2] != s.tables[1][2]
    assert m.num_free_blocks() == 16 - 4


def test_exhausted_pool_raises():
    m = rmlx_kv.PagedCacheManager(4, 2)
    s = SequenceBlocks(m, 4, [8])
    with pytest.raises(PoolExhausted):
        s.append_slots()
    with pytest.raises(PoolExhausted):
        SequenceBlocks(rmlx_kv.PagedCacheManager(4, 1), 4, [5])


def test_release_returns_blocks():
    m = rmlx_kv.PagedCacheManager(4, 8)
    s = SequenceBlocks(m, 4, [9, 0])
    s.fork(0, 1)
    s.release(0)
    assert m.num_free_blocks() == 5 and all(m.ref_count(b) == 1 for b in s.tables[1])
    s.release(1)
    assert m.num_free_blocks() == 8
