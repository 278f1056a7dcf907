"""Host-side mirror of the rmlx-serve-cache types over the C ABI.

Same names, argument meaning and error behaviour as the Rust crate
(crates/rmlx-serve-cache/src): methods that return ``Option`` return
``None``; methods that ``assert!`` raise :class:`RmlxError` with the
reference's panic message.
"""
from __future__ import annotations

import ctypes as C
import weakref
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import check, lib


def _u32(tokens: Sequence[int]):
    a = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
    return a, a.ctypes.data_as(_lib.u32p)


def _i32(ids: Sequence[int]):
    a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
    return a, a.ctypes.data_as(_lib.i32p)


@dataclass
class KVCacheBlock:
    """paged_cache.rs:14-26"""
    block_id: int
    ref_count: int
    hash: Optional[int]
    tokens: List[int]
    num_filled: int

    def is_full(self, block_size: int) -> bool:  # :41-43
        return self.num_filled >= block_size

    def is_empty(self) -> bool:  # :46-48
        return self.num_filled == 0


class PagedCacheManager:
    """paged_cache.rs:71-302"""

    def __init__(self, block_size: int, num_blocks: int):
        h = _lib.vp()
        check(lib.rmlx_block_manager_new(block_size, num_blocks, C.byref(h)))
        self._h = h
        self._bs = block_size
        self._dependents = weakref.WeakSet()  # objects holding references in this manager

    def __del__(self):
        if getattr(self, "_h", None):
            for d in list(getattr(self, "_dependents", ())):
                d.close()  # a batch releases its references before the manager goes
            lib.rmlx_block_manager_destroy(self._h)
            self._h = None

    def allocate(self) -> Optional[int]:
        bid, found = C.c_int32(), C.c_int32()
        check(lib.rmlx_block_manager_allocate(self._h, C.byref(bid), C.byref(found)))
        return bid.value if found.value else None

    def allocate_n(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.int32)
        got = C.c_size_t()
        check(lib.rmlx_block_manager_allocate_n(self._h, n, out.ctypes.data_as(_lib.i32p), C.byref(got)))
        return out[:got.value]

    def free(self, block_id: int) -> None:
        check(lib.rmlx_block_manager_free(self._h, block_id))

    def free_n(self, block_ids: Sequence[int]) -> None:
        a, p = _i32(block_ids)
        check(lib.rmlx_block_manager_free_n(self._h, p, len(a)))

    def ref_count(self, block_id: int) -> int:
        out = C.c_size_t()
        check(lib.rmlx_block_manager_ref_count(self._h, block_id, C.byref(out)))
        return out.value

    def increment_ref(self, block_id: int) -> None:
        check(lib.rmlx_block_manager_increment_ref(self._h, block_id))

    def copy_on_write(self, block_id: int) -> Optional[int]:
        nid, copied = C.c_int32(), C.c_int32()
        check(lib.rmlx_block_manager_copy_on_write(self._h, block_id, C.byref(nid), C.byref(copied)))
        return nid.value if copied.value else None

    def num_free_blocks(self) -> int:
        return lib.rmlx_block_manager_num_free_blocks(self._h)

    def num_allocated_blocks(self) -> int:
        return lib.rmlx_block_manager_num_allocated_blocks(self._h)

    def num_blocks(self) -> int:
        return lib.rmlx_block_manager_num_blocks(self._h)

    def block_size(self) -> int:
        return lib.rmlx_block_manager_block_size(self._h)

    def get_block(self, block_id: int) -> Optional[KVCacheBlock]:
        if block_id < 0:
            return None
        v = _lib.BlockView()
        toks = (C.c_uint32 * max(self._bs, 1))()
        found = C.c_int32()
        check(lib.rmlx_block_manager_get_block(self._h, block_id, C.byref(v), toks, self._bs, C.byref(found)))
        if not found.value:
            return None
        return KVCacheBlock(v.block_id, v.ref_count, v.hash if v.has_hash else None,
                            list(toks[:v.num_filled]), v.num_filled)

    def register_hash(self, block_id: int, hash: int) -> None:
        check(lib.rmlx_block_manager_register_hash(self._h, block_id, hash))

    def lookup_hash(self, hash: int) -> Optional[int]:
        bid, found = C.c_int32(), C.c_int32()
        check(lib.rmlx_block_manager_lookup_hash(self._h, hash, C.byref(bid), C.byref(found)))
        return bid.value if found.value else None

    def append_tokens(self, block_id: int, tokens: Sequence[int]) -> None:
        a, p = _u32(tokens)
        check(lib.rmlx_block_manager_append_tokens(self._h, block_id, p, len(a)))


class PrefixCacheManager:
    """prefix_cache.rs:44-292"""

    def __init__(self, max_blocks: int):
        h = _lib.vp()
        check(lib.rmlx_prefix_cache_new(max_blocks, C.byref(h)))
        self._h = h
        self._dependents = weakref.WeakSet()

    def __del__(self):
        if getattr(self, "_h", None):
            for d in list(getattr(self, "_dependents", ())):
                d.close()
            lib.rmlx_prefix_cache_destroy(self._h)
            self._h = None

    def lookup(self, tokens: Sequence[int]) -> List[int]:
        a, p = _u32(tokens)
        out = np.empty(max(len(a), 1), dtype=np.int32)
        n = C.c_size_t()
        check(lib.rmlx_prefix_cache_lookup(self._h, p, len(a), out.ctypes.data_as(_lib.i32p), C.byref(n)))
        return out[:n.value].tolist()

    def insert(self, tokens: Sequence[int], block_ids: Sequence[int]) -> None:
        a, p = _u32(tokens)
        b, q = _i32(block_ids)
        check(lib.rmlx_prefix_cache_insert(self._h, p, len(a), q, len(b)))

    def evict_lru(self) -> Optional[int]:
        bid, found = C.c_int32(), C.c_int32()
        check(lib.rmlx_prefix_cache_evict_lru(self._h, C.byref(bid), C.byref(found)))
        return bid.value if found.value else None

    def hit_rate(self) -> float:
        return lib.rmlx_prefix_cache_hit_rate(self._h)

    def num_blocks(self) -> int:
        return lib.rmlx_prefix_cache_num_blocks(self._h)

    def max_blocks(self) -> int:
        return lib.rmlx_prefix_cache_max_blocks(self._h)

    def is_full(self) -> bool:
        return bool(lib.rmlx_prefix_cache_is_full(self._h))

    def num_nodes(self) -> int:
        return lib.rmlx_prefix_cache_num_nodes(self._h)


class MemoryAwarePrefixCache:
    """memory.rs:10-200"""

    def __init__(self, max_blocks: int, memory_limit_mb: int, bytes_per_block: Optional[int] = None):
        h = _lib.vp()
        if bytes_per_block is None:
            check(lib.rmlx_mem_prefix_cache_new(max_blocks, memory_limit_mb, C.byref(h)))
        else:
            check(lib.rmlx_mem_prefix_cache_with_block_size(max_blocks, memory_limit_mb, bytes_per_block,
                                                            C.byref(h)))
        self._h = h

    @classmethod
    def with_block_size(cls, max_blocks: int, memory_limit_mb: int, bytes_per_block: int):
        return cls(max_blocks, memory_limit_mb, bytes_per_block)

    def __del__(self):
        if getattr(self, "_h", None):
            lib.rmlx_mem_prefix_cache_destroy(self._h)
            self._h = None

    @staticmethod
    def available_memory_mb() -> int:  # memory.rs:88-91 (non-macOS build)
        return 2 ** 64 - 1

    def should_evict(self) -> bool:
        return bool(lib.rmlx_mem_prefix_cache_should_evict(self._h))

    def evict_until_threshold(self) -> None:
        check(lib.rmlx_mem_prefix_cache_evict_until_threshold(self._h))

    def lookup(self, tokens: Sequence[int]) -> List[int]:
        a, p = _u32(tokens)
        out = np.empty(max(len(a), 1), dtype=np.int32)
        n = C.c_size_t()
        check(lib.rmlx_mem_prefix_cache_lookup(self._h, p, len(a), out.ctypes.data_as(_lib.i32p), C.byref(n)))
        return out[:n.value].tolist()

    def insert(self, tokens: Sequence[int], block_ids: Sequence[int]) -> None:
        a, p = _u32(tokens)
        b, q = _i32(block_ids)
        check(lib.rmlx_mem_prefix_cache_insert(self._h, p, len(a), q, len(b)))

    def evict_lru(self) -> Optional[int]:
        bid, found = C.c_int32(), C.c_int32()
        check(lib.rmlx_mem_prefix_cache_evict_lru(self._h, C.byref(bid), C.byref(found)))
        return bid.value if found.value else None

    def drain_evicted(self) -> List[int]:
        out: List[int] = []
        buf = np.empty(4096, dtype=np.int32)
        n = C.c_size_t()
        while True:
            check(lib.rmlx_mem_prefix_cache_drain_evicted(self._h, buf.ctypes.data_as(_lib.i32p), len(buf),
                                                          C.byref(n)))
            out.extend(buf[:n.value].tolist())
            if n.value < len(buf):
                return out

    def hit_rate(self) -> float:
        return lib.rmlx_mem_prefix_cache_hit_rate(self._h)

    def current_usage_bytes(self) -> int:
        return lib.rmlx_mem_prefix_cache_current_usage_bytes(self._h)

    def memory_limit_bytes(self) -> int:
        return lib.rmlx_mem_prefix_cache_memory_limit_bytes(self._h)

    def num_blocks(self) -> int:
        return lib.rmlx_mem_prefix_cache_num_blocks(self._h)


class QuantizedKVCache:
    """quantized_cache.rs:14-296, storage and (de)quantisation on a GPU."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, bits: int, group_size: int,
                 device: int = 0):
        h = _lib.vp()
        check(lib.rmlx_qcache_new(num_layers, num_kv_heads, head_dim, bits, group_size, device, C.byref(h)))
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None):
            lib.rmlx_qcache_destroy(self._h)
            self._h = None

    def append(self, layer: int, keys, values, new_tokens: int) -> None:
        k = np.ascontiguousarray(np.asarray(keys, dtype=np.float32))
        v = np.ascontiguousarray(np.asarray(values, dtype=np.float32))
        if k.size != v.size:
            raise _lib.RmlxError(_lib.E_BAD_ARG, f"values length mismatch: expected {k.size}, got {v.size}")
        check(lib.rmlx_qcache_append(self._h, layer, k.ctypes.data_as(_lib.f32p), v.ctypes.data_as(_lib.f32p),
                                     k.size, new_tokens))

    def _get(self, fn, layer: int) -> np.ndarray:
        n = C.c_size_t()
        check(fn(self._h, layer, None, 0, C.byref(n)))
        out = np.empty(n.value, dtype=np.float32)
        if n.value:
            check(fn(self._h, layer, out.ctypes.data_as(_lib.f32p), n.value, C.byref(n)))
        return out

    def get_keys_dequantized(self, layer: int) -> np.ndarray:
        return self._get(lib.rmlx_qcache_get_keys_dequantized, layer)

    def get_values_dequantized(self, layer: int) -> np.ndarray:
        return self._get(lib.rmlx_qcache_get_values_dequantized, layer)

    def raw(self, layer: int, which: int):
        """Stored (bytes, scales, zeros) of keys (which=0) or values (1)."""
        nb, ng = C.c_size_t(), C.c_size_t()
        check(lib.rmlx_qcache_raw(self._h, layer, which, None, 0, None, None, 0, C.byref(nb), C.byref(ng)))
        b = np.empty(nb.value, dtype=np.uint8)
        s = np.empty(ng.value, dtype=np.float32)
        z = np.empty(ng.value, dtype=np.float32)
        check(lib.rmlx_qcache_raw(self._h, layer, which, b.ctypes.data_as(_lib.u8p), nb.value,
                                  s.ctypes.data_as(_lib.f32p), z.ctypes.data_as(_lib.f32p), ng.value,
                                  C.byref(nb), C.byref(ng)))
        return b, s, z

    def seq_len(self) -> int:
        return lib.rmlx_qcache_seq_len(self._h)

    def num_layers(self) -> int:
        return lib.rmlx_qcache_num_layers(self._h)

    def bits(self) -> int:
        return lib.rmlx_qcache_bits(self._h)

    def group_size(self) -> int:
        return lib.rmlx_qcache_group_size(self._h)


def prefix_admit(mgr: PagedCacheManager, prefix: PrefixCacheManager, tokens, cu_tokens, hashes, cu_blocks):
    """Admit requests in order through `mgr` and `prefix` (rmlx_prefix_admit).

    Returns (block_ids per block, evicted block ids in order, stats dict).
    """
    t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32)) if len(tokens) else np.zeros(1, np.uint32)
    cu = np.ascontiguousarray(np.asarray(cu_tokens, dtype=np.int64))
    cub = np.ascontiguousarray(np.asarray(cu_blocks, dtype=np.int64))
    hs = np.ascontiguousarray(np.asarray(hashes, dtype=np.uint64)) if len(hashes) else np.zeros(1, np.uint64)
    nblk = int(cub[-1])
    ids = np.zeros(max(nblk, 1), dtype=np.int32)
    cap = 4 * nblk + 16
    ev = np.zeros(cap, dtype=np.int32)
    nev = C.c_size_t()
    stats = _lib.AdmitStats()
    check(lib.rmlx_prefix_admit(mgr._h, prefix._h, t.ctypes.data_as(_lib.u32p), cu.ctypes.data_as(_lib.i64p),
                                hs.ctypes.data_as(_lib.u64p), cub.ctypes.data_as(_lib.i64p), len(cu) - 1,
                                ids.ctypes.data_as(_lib.i32p), ev.ctypes.data_as(_lib.i32p), cap, C.byref(nev),
                                C.byref(stats)))
    st = {n: getattr(stats, n) for n, _ in _lib.AdmitStats._fields_}
    return ids[:nblk], ev[:min(nev.value, cap)], st
