"""The batch planner (rmlx_kv_batch_*) against its restatement over the
oracle's block manager, prefix trie and XXH64 (tests/batch_model.py):
random admissions, steps, forks and removals give the same rows, cached
token counts, slots, copy-on-write pairs, block tables, reference counts,
free lists and statistics."""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from batch_model import BatchModel, Exhausted
from rmlx_kv.batch import KVBatch


def _same_state(pm, om, nb):
    for b in range(nb):
        assert pm.ref_count(b) == om.ref_count(b)
    assert pm.num_free_blocks() == om.num_free_blocks()


@pytest.mark.parametrize("seed,prefix,bs,nb", [(0, True, 16, 200), (1, True, 4, 60), (2, False, 16, 120),
                                               (3, True, 8, 40), (4, True, 1, 90)])
def test_planner_matches_restatement(seed, prefix, bs, nb):
    rng = np.random.default_rng(500 + seed)
    pm, om = rmlx_kv.PagedCacheManager(bs, nb), orc.PagedCacheManager(bs, nb)
    pp = rmlx_kv.PrefixCacheManager(nb) if prefix else None
    op = orc.PrefixCacheManager(nb) if prefix else None
    batch, model = KVBatch(pm, pp, 8), BatchModel(om, op, 8, bs)
    prompts = [rng.integers(0, 50, size=int(rng.integers(1, 60))).tolist() for _ in range(4)]
    live, uid = [], 0
    for _ in range(300):
        r = rng.random()
        if r < 0.2:
            base = prompts[int(rng.integers(len(prompts)))]
            prompt = base[:int(rng.integers(1, len(base) + 1))] + rng.integers(0, 50, size=int(rng.integers(0, 9))).tolist()
            uid += 1
            try:
                want = model.add(uid, prompt)
            except Exhausted:
                with pytest.raises(rmlx_kv.RmlxError):
                    batch.add(uid, prompt)
            else:
                row, cached, slots = batch.add(uid, prompt)
                assert (row, cached, slots.tolist()) == (want[0], want[1], want[2])
                live.append(uid)
        elif r < 0.3 and live:
            parent = live[int(rng.integers(len(live)))]
            uid += 1
            try:
                want = model.fork(parent, uid)
            except Exhausted:
                with pytest.raises(rmlx_kv.RmlxError):
                    batch.fork(parent, uid)
            else:
                assert batch.fork(parent, uid) == want
                live.append(uid)
        elif r < 0.42 and live:
            u = live.pop(int(rng.integers(len(live))))
            cache = bool(rng.random() < 0.7)
            model.remove(u, cache)
            batch.remove(u, cache)
        elif live:
            uids = [u for u in live if rng.random() < 0.8]
            toks = rng.integers(0, 50, size=len(uids)).tolist()
            try:
                want = model.step(uids, toks)
            except Exhausted:
                with pytest.raises(rmlx_kv.RmlxError):
                    batch.step(uids, toks)
            else:
                slots, src, dst = batch.step(uids, toks)
                assert slots.tolist() == want[0] and src.tolist() == want[1] and dst.tolist() == want[2]
        bt, lens = batch.tables()
        wbt, wlens = model.tables()
        np.testing.assert_array_equal(lens, wlens)
        np.testing.assert_array_equal(bt, wbt)
        _same_state(pm, om, nb)
    assert batch.stats() == model.stats
    if prefix:
        assert batch.stats()["cached_tokens"] > 0
    batch.close()


def test_prefix_reuse_and_copy_on_write():
    m, p = rmlx_kv.PagedCacheManager(4, 32), rmlx_kv.PrefixCacheManager(32)
    b = KVBatch(m, p, 4)
    prompt = list(range(10))
    _, c0, s0 = b.add(1, prompt)
    assert c0 == 0 and len(s0) == 10
    _, c1, s1 = b.add(2, prompt)
    assert c1 == 8 and len(s1) == 2  # two full blocks reused, the tail recomputed
    b.fork(1, 3)  # shares block 2 (2 of 4 rows filled)
    slots, src, dst = b.step([1, 3], [5, 5])
    assert len(src) == 1  # sequence 1 writes the shared tail first and takes the copy
    _, ln, ids = b.seq(3)
    assert ln == 11 and src[0] == ids[2]
    with pytest.raises(rmlx_kv.RmlxError, match="listed twice"):
        b.step([1, 1], [0, 0])
    with pytest.raises(rmlx_kv.RmlxError, match="empty prompt"):
        b.add(9, [])
    with pytest.raises(rmlx_kv.RmlxError, match="already"):
        b.add(1, [1])
    b.close()
    assert m.num_free_blocks() == 32 - p.num_blocks()


def test_full_prompt_hit_still_computes_last_token():
    m, p = rmlx_kv.PagedCacheManager(4, 16), rmlx_kv.PrefixCacheManager(16)
    b = KVBatch(m, p, 2)
    b.add(1, list(range(8)))
    b.remove(1, True)
    _, cached, slots = b.add(2, list(range(8)))  # both blocks cached, but the last token is recomputed
    assert cached == 4 and len(slots) == 4
    b.close()


def test_exhaustion_is_all_or_nothing():
    m = rmlx_kv.PagedCacheManager(2, 3)
    b = KVBatch(m, None, 4)
    b.add(1, [1, 2])
    b.add(2, [3, 4])
    before = b.tables()
    with pytest.raises(rmlx_kv.RmlxError):
        b.step([1, 2], [5, 6])  # needs 2 new blocks, 1 free
    after = b.tables()
    np.testing.assert_array_equal(before[0], after[0])
    np.testing.assert_array_equal(before[1], after[1])
    assert m.num_free_blocks() == 1
    b.close()


def test_batch_kv_cache_mapping():
    """The reference's BatchKVCache tests (batch_cache.rs:120-197) through
    the calls that replace it: insert -> add (the batch picks the lowest
    free row), get/get_mut -> seq, remove -> remove, active_count ->
    num_active, iter -> rows, capacity -> max_seqs.  compact has nothing to
    move: rows are block-table rows, and a free row is a zero-length row."""
    m = rmlx_kv.PagedCacheManager(4, 64)
    b = KVBatch(m, None, 4)
    assert b.max_seqs == 4 and b.num_active() == 0
    # insert at 0, 1, 2 (lowest free rows), then remove 0: rows 1 and 2 live
    for uid in (10, 11, 12):
        row, cached, slots = b.add(uid, [1, 2, 3])
        assert row == uid - 10 and cached == 0 and len(slots) == 3
    b.remove(10)
    assert b.num_active() == 2
    uids, live = b.rows()
    assert list(np.flatnonzero(live)) == [1, 2] and list(uids) == [0, 11, 12, 0]
    with pytest.raises(rmlx_kv.RmlxError):
        b.seq(10)  # removed: get(0) is None
    assert b.seq(11)[0] == 1
    with pytest.raises(rmlx_kv.RmlxError):
        b.remove(10)  # remove of an empty slot
    bt, lens = b.tables()
    assert list(lens) == [0, 3, 3]  # rows up to the last live one; the gap is a zero-length row
    # the next admission takes the gap
    assert b.add(13, [4])[0] == 0
    b.add(14, [5])
    with pytest.raises(rmlx_kv.RmlxError):
        b.add(15, [6])  # capacity 4 exceeded
    assert b.num_active() == 4
    b.close()
    assert m.num_free_blocks() == 64
