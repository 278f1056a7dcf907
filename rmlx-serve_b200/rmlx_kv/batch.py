"""Block tables of a decode batch with forked sequences (beam / speculative
branches), kept over a block manager.

A fork makes the child share every block of the parent: the child's old
blocks are released (paged_cache.rs:125-149, free) and each of the
parent's gains a reference (paged_cache.rs:172-182, increment_ref).  The
next token appended to a sequence whose tail block is shared goes through
copy_on_write (paged_cache.rs:197-224): the manager hands out a private block, and the
device must copy the shared tile into it (``KVPool.copy_blocks``) before
the token is written.  ``append_slots`` returns those copy pairs together
with the slot of each sequence's new token, so one step is

    copy_blocks(cow_src, cow_dst) -> append(slots) -> gather(block_table)

The manager is any object with the reference's allocate / free /
increment_ref / copy_on_write methods (this package's PagedCacheManager,
or the oracle's restatement in the tests).
"""
from __future__ import annotations

import ctypes as C
from typing import List, Sequence, Tuple

import numpy as np

from . import _lib


class PoolExhausted(RuntimeError):
    pass


class SequenceBlocks:
    def __init__(self, mgr, block_size: int, lens: Sequence[int]):
        self.mgr = mgr
        self.bs = int(block_size)
        self.lens = [int(x) for x in lens]
        self.tables: List[List[int]] = [[self._alloc() for _ in range((n + self.bs - 1) // self.bs)]
                                        for n in self.lens]

    def _alloc(self) -> int:
        bid = self.mgr.allocate()
        if bid is None:
            raise PoolExhausted("no free block")
        return int(bid)

    def release(self, seq: int) -> None:
        """Drop the sequence's references (its blocks return to the free list
        when no other sequence holds them)."""
        for b in self.tables[seq]:
            self.mgr.free(b)
        self.tables[seq] = []
        self.lens[seq] = 0

    def fork(self, parent: int, child: int) -> None:
        """Replace `child` by a branch of `parent` that shares all its blocks."""
        if parent == child:
            return
        self.release(child)
        for b in self.tables[parent]:
            self.mgr.increment_ref(b)
        self.tables[child] = list(self.tables[parent])
        self.lens[child] = self.lens[parent]

    def append_slots(self) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        """One new token per sequence.  Returns (cow_src, cow_dst, slots):
        the tiles to copy before the append and each token's pool slot
        (block * block_size + offset)."""
        src, dst = [], []
        slots = np.empty(len(self.lens), dtype=np.int32)
        for s, pos in enumerate(self.lens):
            t = self.tables[s]
            bi = pos // self.bs
            if bi == len(t):
                t.append(self._alloc())
            else:
                nid = self.mgr.copy_on_write(t[bi])
                if nid is not None:
                    src.append(t[bi])
                    dst.append(int(nid))
                    t[bi] = int(nid)
            slots[s] = t[bi] * self.bs + pos % self.bs
            self.lens[s] = pos + 1
        return np.array(src, dtype=np.int32), np.array(dst, dtype=np.int32), slots

    def trim(self, seq: int, n: int) -> List[int]:
        """Drop the last n tokens of `seq` (all of them when n >= its length,
        as trim_prompt_cache, prompt_cache.rs:218-226); blocks that no longer
        hold a token lose this sequence's reference.  Returns those blocks."""
        keep = max(self.lens[seq] - int(n), 0)
        nb = (keep + self.bs - 1) // self.bs
        dropped = self.tables[seq][nb:]
        for b in dropped:
            self.mgr.free(b)
        self.tables[seq] = self.tables[seq][:nb]
        self.lens[seq] = keep
        return dropped

    def block_table(self) -> np.ndarray:
        """[num_seqs, max blocks] int32, rows padded with 0."""
        width = max([len(t) for t in self.tables] + [1])
        bt = np.zeros((len(self.tables), width), dtype=np.int32)
        for s, t in enumerate(self.tables):
            bt[s, :len(t)] = t
        return bt

    def seq_lens(self) -> np.ndarray:
        return np.array(self.lens, dtype=np.int32)


class RotatingBlocks:
    """One sliding-window sequence as a ring over its blocks: the
    (written, offset) state machine of RotatingKVCache (rotating_cache.rs:
    16-283) kept by the library (rmlx_rotating_* in the C ABI), with ring
    position p stored in block table entry p / block_size, row
    p % block_size.  Blocks are taken from the manager (this package's
    PagedCacheManager) as the ring first reaches them; the reference
    preallocates max_size rows.

    The state advances once per token for all layers of the pool; the
    reference advances it on every per-layer append call, which is the same
    for a one-layer cache (its tests) and for each layer driven as its own
    cache.  The reference's panics (keep >= max_size, trimming more than is
    trimmable) raise ValueError here.
    """

    def __init__(self, mgr, block_size: int, max_size: int, keep: int):
        h = _lib.vp()
        rc = _lib.lib.rmlx_rotating_new(mgr._h, block_size, max_size, keep, C.byref(h))
        if rc == _lib.RMLX_E_BAD_ARG:
            raise ValueError(_lib.lib.rmlx_last_error().decode())
        _lib.check(rc)
        self._h, self._mgr = h, mgr
        self.bs, self.max_size, self.keep = int(block_size), int(max_size), int(keep)
        mgr._dependents.add(self)

    def __del__(self):
        self.close()

    def close(self):
        """Return the ring's blocks to the manager and drop the ring."""
        if getattr(self, "_h", None):
            # When a garbage-collected cycle took the manager first, its
            # blocks are gone with it: only the ring's own memory is left.
            if getattr(self._mgr, "_h", None):
                _lib.lib.rmlx_rotating_destroy(self._h)
            self._h = None

    @property
    def table(self) -> List[int]:
        """The ring's blocks, in ring order."""
        n = C.c_int32()
        _lib.check(_lib.lib.rmlx_rotating_blocks(self._h, None, 0, C.byref(n)))
        out = np.zeros(max(n.value, 1), np.int32)
        _lib.check(_lib.lib.rmlx_rotating_blocks(self._h, out.ctypes.data_as(_lib.i32p), len(out), C.byref(n)))
        return out[:n.value].tolist()

    @property
    def written(self) -> int:
        return int(_lib.lib.rmlx_rotating_written(self._h))

    def append_slots(self, n: int) -> np.ndarray:
        """Slots of n new tokens in order (append, :94-143).  A ring position
        written twice within the call keeps the later token: the earlier
        token's slot is -1 (skipped by rmlx_kv_append).  Raises
        PoolExhausted, with the state unchanged, when the blocks the tokens
        reach cannot be had."""
        slots = np.empty(max(n, 1), dtype=np.int32)
        rc = _lib.lib.rmlx_rotating_append_slots(self._h, n, slots.ctypes.data_as(_lib.i32p))
        if rc == _lib.RMLX_E_EXHAUSTED:
            raise PoolExhausted(_lib.lib.rmlx_last_error().decode())
        _lib.check(rc)
        return slots[:n]

    def seq_len(self) -> int:  # :201-203
        return int(_lib.lib.rmlx_rotating_seq_len(self._h))

    def can_trim(self) -> bool:  # :253-255
        return bool(_lib.lib.rmlx_rotating_can_trim(self._h))

    def ring_offset(self) -> int:
        """For rmlx_kv_gather_ring: -1 before the ring has rotated
        (written <= max_size), else the offset of its oldest row."""
        return int(_lib.lib.rmlx_rotating_ring_offset(self._h))

    def trim(self, n: int):
        """Drop the n oldest rows after `keep` (trim, :213-247).  Before the
        ring rotates the rows above them shift down: returns the (src, dst)
        slot lists that rmlx_kv_move_rows must apply; after, only the state
        moves (empty lists)."""
        src = np.empty(max(self.max_size, 1), np.int32)
        dst = np.empty_like(src)
        nm = C.c_int32()
        rc = _lib.lib.rmlx_rotating_trim(self._h, n, src.ctypes.data_as(_lib.i32p), dst.ctypes.data_as(_lib.i32p),
                                         len(src), C.byref(nm))
        if rc in (_lib.RMLX_E_RANGE, _lib.RMLX_E_BAD_ARG):
            raise ValueError(_lib.lib.rmlx_last_error().decode())
        _lib.check(rc)
        return src[:nm.value].copy(), dst[:nm.value].copy()

    def release(self) -> None:
        """Return the ring's blocks to the manager; the ring starts empty."""
        _lib.lib.rmlx_rotating_release(self._h)


class KVBatch:
    """The scheduler's KV bookkeeping on block tables (rmlx_kv_batch_* in
    the C ABI): admit prompts (reusing prefix-cache blocks), one token per
    sequence per step (with copy-on-write of shared tails), forks, removal
    (optionally into the prefix cache), and the dense block tables and
    lengths a step's device calls take."""

    def __init__(self, mgr, prefix=None, max_seqs: int = 256):
        h = _lib.vp()
        _lib.check(_lib.lib.rmlx_kv_batch_new(mgr._h, prefix._h if prefix is not None else None, max_seqs,
                                              C.byref(h)))
        self._h, self._mgr, self._prefix, self.max_seqs = h, mgr, prefix, max_seqs
        mgr._dependents.add(self)
        if prefix is not None:
            prefix._dependents.add(self)

    def __del__(self):
        self.close()

    def close(self):
        if getattr(self, "_h", None):
            # When a garbage-collected cycle took the manager or the prefix
            # cache first (their weak references to this batch were cleared
            # before it could be closed), the references it held went with
            # them: destroying the batch would touch freed state.
            alive = getattr(self._mgr, "_h", None) and (self._prefix is None or getattr(self._prefix, "_h", None))
            if alive:
                _lib.lib.rmlx_kv_batch_destroy(self._h)
            self._h = None

    def add(self, uid: int, prompt: Sequence[int]):
        """-> (row, cached_tokens, slots of the uncached prompt tokens)."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        slots = np.empty(max(len(p), 1), dtype=np.int32)
        row, cached = C.c_int32(), C.c_int32()
        _lib.check(_lib.lib.rmlx_kv_batch_add(self._h, uid, p.ctypes.data_as(_lib.u32p), len(p), C.byref(row),
                                              C.byref(cached), slots.ctypes.data_as(_lib.i32p)))
        return row.value, cached.value, slots[:len(p) - cached.value]

    def fork(self, parent: int, child: int) -> int:
        row = C.c_int32()
        _lib.check(_lib.lib.rmlx_kv_batch_fork(self._h, parent, child, C.byref(row)))
        return row.value

    def remove(self, uid: int, cache_prefix: bool = False) -> None:
        _lib.check(_lib.lib.rmlx_kv_batch_remove(self._h, uid, int(cache_prefix)))

    def step(self, uids: Sequence[int], tokens: Sequence[int]):
        """-> (slots, cow_src, cow_dst) for one token per listed sequence."""
        u = np.ascontiguousarray(np.asarray(uids, dtype=np.uint64))
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        if len(u) != len(t):
            raise ValueError("one token per sequence")
        n = len(u)
        slots = np.empty(max(n, 1), np.int32)
        src = np.empty(max(n, 1), np.int32)
        dst = np.empty(max(n, 1), np.int32)
        nc = C.c_int32()
        _lib.check(_lib.lib.rmlx_kv_batch_step(self._h, u.ctypes.data_as(C.POINTER(C.c_uint64)),
                                               t.ctypes.data_as(_lib.u32p), n, slots.ctypes.data_as(_lib.i32p),
                                               src.ctypes.data_as(_lib.i32p), dst.ctypes.data_as(_lib.i32p),
                                               C.byref(nc)))
        return slots[:n], src[:nc.value], dst[:nc.value]

    def tables(self):
        """-> (block_tables [rows, max_blocks] int32, seq_lens [rows] int32)."""
        nr, mb = C.c_int32(), C.c_int32()
        _lib.check(_lib.lib.rmlx_kv_batch_tables(self._h, None, 0, None, 0, C.byref(nr), C.byref(mb)))
        bt = np.zeros((max(nr.value, 1), max(mb.value, 1)), np.int32)
        lens = np.zeros(max(nr.value, 1), np.int32)
        _lib.check(_lib.lib.rmlx_kv_batch_tables(self._h, bt.ctypes.data_as(_lib.i32p), bt.shape[1],
                                                 lens.ctypes.data_as(_lib.i32p), bt.shape[0], C.byref(nr),
                                                 C.byref(mb)))
        return bt[:nr.value, :mb.value], lens[:nr.value]

    def seq(self, uid: int):
        """-> (row, length, block ids) of one sequence."""
        row, ln, nb = C.c_int32(), C.c_int32(), C.c_int32()
        _lib.check(_lib.lib.rmlx_kv_batch_seq(self._h, uid, C.byref(row), C.byref(ln), None, 0, C.byref(nb)))
        ids = np.zeros(max(nb.value, 1), np.int32)
        _lib.check(_lib.lib.rmlx_kv_batch_seq(self._h, uid, C.byref(row), C.byref(ln), ids.ctypes.data_as(_lib.i32p),
                                              len(ids), C.byref(nb)))
        return row.value, ln.value, ids[:nb.value]

    def num_active(self) -> int:
        """Live sequences (BatchKVCache::active_count)."""
        return int(_lib.lib.rmlx_kv_batch_num_active(self._h))

    def rows(self):
        """-> uids [max_seqs] uint64 (0 for a free row) and a live mask
        (BatchKVCache::iter over (row, sequence))."""
        uids = np.zeros(self.max_seqs, np.uint64)
        live = np.zeros(self.max_seqs, np.int32)
        n = C.c_int32()
        _lib.check(_lib.lib.rmlx_kv_batch_rows(self._h, uids.ctypes.data_as(C.POINTER(C.c_uint64)),
                                               live.ctypes.data_as(_lib.i32p), self.max_seqs, C.byref(n)))
        return uids[:n.value], live[:n.value].astype(bool)

    def stats(self) -> dict:
        s = _lib.BatchStats()
        _lib.lib.rmlx_kv_batch_stats(self._h, s)
        return {n: getattr(s, n) for n, _ in s._fields_}
