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


def test_exhausted_pool_leaves_ring_unchanged():
    """append_slots takes every block the new tokens reach before changing
    any state: with too few free blocks it fails and the ring is as before."""
    from rmlx_kv.batch import PoolExhausted
    m = rmlx_kv.PagedCacheManager(4, 3)
    rb = RotatingBlocks(m, 4, 16, 2)
    rb.append_slots(5)  # 2 blocks
    before = (rb.seq_len(), rb.written, rb.ring_offset(), rb.table, m.num_free_blocks())
    with pytest.raises(PoolExhausted):
        rb.append_slots(8)  # reaches position 12: 4 blocks
    assert (rb.seq_len(), rb.written, rb.ring_offset(), rb.table, m.num_free_blocks()) == before
    assert len(rb.append_slots(7)) == 7  # up to position 11: the third block
    assert m.num_free_blocks() == 0


def test_trim_reports_moves_and_rejects_short_buffers():
    import ctypes as C
    from rmlx_kv import _lib
    m = rmlx_kv.PagedCacheManager(4, 8)
    rb = RotatingBlocks(m, 4, 10, 1)
    rb.append_slots(7)
    nm = C.c_int32()
    buf = np.zeros(8, np.int32)
    p = buf.ctypes.data_as(_lib.i32p)
    # 7 rows, keep 1, trim 2: rows 3..6 move to 1..4; a 3-entry buffer is short
    assert _lib.lib.rmlx_rotating_trim(rb._h, 2, p, p, 3, C.byref(nm)) == _lib.RMLX_E_BAD_ARG
    assert nm.value == 4 and rb.seq_len() == 7
    src, dst = rb.trim(2)
    assert len(src) == 4 and rb.seq_len() == 5
    t = rb.table
    assert list(src) == [t[p // 4] * 4 + p % 4 for p in range(3, 7)]
    assert list(dst) == [t[p // 4] * 4 + p % 4 for p in range(1, 5)]


def test_ring_closes_before_its_manager():
    m = rmlx_kv.PagedCacheManager(2, 8)
    rb = RotatingBlocks(m, 2, 6, 0)
    rb.append_slots(6)
    assert m.num_free_blocks() == 5
    del m  # the ring still holds the manager; closing the ring frees its blocks
    mgr = rb._mgr
    rb.close()
    assert mgr.num_free_blocks() == 8


def test_ring_c_abi_argument_checks():
    """The C ABI's own checks: a block size other than the manager's, NULL
    outputs, negative counts, and a trim past what is trimmable (the
    reference's panic) leave the ring as it was."""
    import ctypes as C
    from rmlx_kv import _lib
    lib = _lib.lib
    m = rmlx_kv.PagedCacheManager(4, 16)
    h = _lib.vp()
    assert lib.rmlx_rotating_new(m._h, 8, 10, 2, C.byref(h)) == _lib.RMLX_E_BAD_ARG  # manager uses 4
    assert lib.rmlx_rotating_new(m._h, 4, 10, -1, C.byref(h)) == _lib.RMLX_E_BAD_ARG
    rb = RotatingBlocks(m, 4, 10, 2)
    assert lib.rmlx_rotating_append_slots(rb._h, -1, None) == _lib.RMLX_E_BAD_ARG
    assert lib.rmlx_rotating_append_slots(rb._h, 3, None) == _lib.RMLX_E_BAD_ARG
    assert lib.rmlx_rotating_append_slots(rb._h, 0, None) == _lib.RMLX_OK
    rb.append_slots(5)
    n = C.c_int32()
    assert lib.rmlx_rotating_trim(rb._h, 4, None, None, 0, C.byref(n)) == _lib.RMLX_E_RANGE
    assert lib.rmlx_rotating_trim(rb._h, -1, None, None, 0, C.byref(n)) == _lib.RMLX_E_BAD_ARG
    assert lib.rmlx_rotating_blocks(rb._h, None, 0, C.byref(n)) == _lib.RMLX_OK and n.value == 2
    assert rb.seq_len() == 5 and rb.written == 5 and rb.ring_offset() == -1
    assert lib.rmlx_rotating_max_size(rb._h) == 10 and lib.rmlx_rotating_keep(rb._h) == 2
