"""Sliding-window ring over block tables, host logic (no GPU).

RotatingBlocks turns RotatingKVCache's state machine (rotating_cache.rs:
94-262) into slot mappings and row moves.  Simulating the pool as a map
slot -> value, the rows read back in logical order (ring_offset and the
mapping rmlx_kv_gather_ring applies) must equal the oracle's get_keys after
every random append / trim, including appends that wrap the ring within one
call and the reference's state after trimming a rotated ring."""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from rmlx_kv.batch import RotatingBlocks


def _logical(rb, pool):
    L, off, R, keep = rb.seq_len(), rb.ring_offset(), rb.max_size - rb.keep, rb.keep
    out = []
    for i in range(L):
        p = i if (off < 0 or i < keep) else keep + (off + i - keep) % R
        out.append(pool.get(rb.table[p // rb.bs] * rb.bs + p % rb.bs, 0.0))
    return out


@pytest.mark.parametrize("seed", range(6))
def test_ring_matches_rotating_cache(seed):
    rng = np.random.default_rng(900 + seed)
    for _ in range(40):
        max_size = int(rng.integers(2, 48))
        keep = int(rng.integers(0, max_size))
        bs = int(rng.integers(1, 9))
        m = rmlx_kv.PagedCacheManager(bs, 64)
        rb = RotatingBlocks(m, bs, max_size, keep)
        ref = orc.RotatingKVCache(1, 1, 1, max_size, keep)
        pool, val = {}, 1.0
        for _ in range(30):
            if rng.random() < 0.25 and rb.can_trim():
                n = int(rng.integers(0, rb.seq_len() - keep + 1))
                src, dst = rb.trim(n)
                ref.trim(n)
                moved = [pool.get(int(s), 0.0) for s in src]  # all read before any is written
                for d, v in zip(dst, moved):
                    pool[int(d)] = v
            else:
                n = int(rng.integers(1, 2 * max_size))
                ks = np.arange(val, val + n, dtype=np.float32)
                val += n
                slots = rb.append_slots(n)
                ref.append(0, ks, ks, n)
                assert len(set(int(s) for s in slots if s >= 0)) == int((slots >= 0).sum())
                for s, v in zip(slots, ks):
                    if s >= 0:
                        pool[int(s)] = float(v)
            assert rb.seq_len() == ref.seq_len() and rb.can_trim() == (ref.seq_len() > keep)
            assert _logical(rb, pool) == ref.get_keys(0)[0]
        assert len(rb.table) <= -(-max_size // bs)
        rb.release()
        assert m.num_free_blocks() == 64


def test_reference_unit_tests():
    """rotating_cache.rs:300-366 on the ring (1 layer, 1 head, head_dim 1)."""
    m = rmlx_kv.PagedCacheManager(2, 16)
    rb = RotatingBlocks(m, 2, 3, 1)
    pool = {}
    for i in range(3):
        pool[int(rb.append_slots(1)[0])] = float(i + 1)
    assert _logical(rb, pool) == [1.0, 2.0, 3.0]
    pool[int(rb.append_slots(1)[0])] = 4.0
    assert rb.seq_len() == 3 and _logical(rb, pool) == [1.0, 3.0, 4.0]
    rb2 = RotatingBlocks(m, 2, 8, 2)
    pool2 = {}
    for i in range(6):
        pool2[int(rb2.append_slots(1)[0])] = float(i + 1)
    assert rb2.can_trim()
    src, dst = rb2.trim(2)
    moved = [pool2[int(s)] for s in src]
    for d, v in zip(dst, moved):
        pool2[int(d)] = v
    assert rb2.seq_len() == 4 and _logical(rb2, pool2) == [1.0, 2.0, 5.0, 6.0]
    with pytest.raises(ValueError, match="keep \\(5\\) must be less than max_size \\(5\\)"):
        RotatingBlocks(m, 2, 5, 5)
    with pytest.raises(ValueError, match="cannot trim"):
        rb2.trim(3)
