"""ORACLE -- TEST INFRASTRUCTURE ONLY.

ctypes binding of oracle/_build/libkv_oracle.so, the CPU restatement of the
rmlx-serve-cache crate (see kv_oracle.cc for the file:line of every
function).  Only tests/, __graft_entry__.smoke() and the CPU-baseline leg of
bench.py import this module; the product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import List, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libkv_oracle.so")


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


if not os.path.exists(LIB_PATH):
    build()
_l = C.CDLL(LIB_PATH)

sz = C.c_size_t
szp = C.POINTER(C.c_size_t)
vp = C.c_void_p
i32p = C.POINTER(C.c_int32)
i64p = C.POINTER(C.c_int64)
u32p = C.POINTER(C.c_uint32)
u64p = C.POINTER(C.c_uint64)
u8p = C.POINTER(C.c_uint8)
f32p = C.POINTER(C.c_float)
ip = C.POINTER(C.c_int)


def _sig(name, res, *args):
    f = getattr(_l, name)
    f.restype = res
    f.argtypes = list(args)


_sig("orc_mgr_new", vp, sz, sz)
_sig("orc_mgr_delete", None, vp)
_sig("orc_mgr_allocate", C.c_int, vp, szp)
_sig("orc_mgr_free", C.c_int, vp, sz)
_sig("orc_mgr_ref_count", C.c_int, vp, sz, szp)
_sig("orc_mgr_increment_ref", C.c_int, vp, sz)
_sig("orc_mgr_copy_on_write", C.c_int, vp, sz, szp, ip)
_sig("orc_mgr_num_free", sz, vp)
_sig("orc_mgr_num_allocated", sz, vp)
_sig("orc_mgr_register_hash", C.c_int, vp, sz, C.c_uint64)
_sig("orc_mgr_lookup_hash", C.c_int, vp, C.c_uint64, szp)
_sig("orc_mgr_append_tokens", C.c_int, vp, sz, u32p, sz)
_sig("orc_mgr_get_block", C.c_int, vp, sz, szp, ip, u64p, szp, u32p, sz, szp)
_sig("orc_prefix_new", vp, sz)
_sig("orc_prefix_delete", None, vp)
_sig("orc_prefix_lookup", sz, vp, u32p, sz, szp, sz)
_sig("orc_prefix_insert", None, vp, u32p, sz, szp, sz)
_sig("orc_prefix_evict_lru", C.c_int, vp, szp)
_sig("orc_prefix_insert_report", None, vp, u32p, sz, szp, sz, C.POINTER(C.c_int32), i64p)
_sig("orc_prefix_hit_rate", C.c_double, vp)
_sig("orc_prefix_num_blocks", sz, vp)
_sig("orc_prefix_num_nodes", sz, vp)
_sig("orc_mem_new", vp, sz, sz, sz)
_sig("orc_mem_delete", None, vp)
_sig("orc_mem_insert", None, vp, u32p, sz, szp, sz)
_sig("orc_mem_lookup", sz, vp, u32p, sz, szp, sz)
_sig("orc_mem_evict_lru", C.c_int, vp, szp)
_sig("orc_mem_should_evict", C.c_int, vp)
_sig("orc_mem_usage", sz, vp)
_sig("orc_mem_limit", sz, vp)
_sig("orc_mem_num_blocks", sz, vp)
_sig("orc_mem_evicted", sz, vp, szp, sz)
_sig("orc_quantize_group", sz, f32p, sz, C.c_int, u8p, f32p, f32p)
_sig("orc_dequantize_group", sz, u8p, sz, C.c_float, C.c_float, C.c_int, f32p)
_sig("orc_qcache_new", vp, sz, sz, sz, C.c_int, sz)
_sig("orc_qcache_delete", None, vp)
_sig("orc_qcache_append", C.c_int, vp, sz, f32p, f32p, sz, sz)
_sig("orc_qcache_seq_len", sz, vp)
_sig("orc_qcache_get_dequantized", C.c_int, vp, sz, C.c_int, f32p, sz, szp)
_sig("orc_qcache_raw", sz, vp, sz, C.c_int, u8p, sz, f32p, f32p, sz, szp)
_sig("orc_rot_new", vp, sz, sz, sz, sz, sz)
_sig("orc_rot_delete", None, vp)
_sig("orc_rot_append", C.c_int, vp, sz, f32p, f32p, sz, sz)
_sig("orc_rot_seq_len", sz, vp)
_sig("orc_rot_get", None, vp, sz, C.c_int, f32p)
_sig("orc_rot_trim", C.c_int, vp, sz)
_sig("orc_xxh64", C.c_uint64, u8p, sz, C.c_uint64)
_sig("orc_hash_chains", None, u32p, i64p, u64p, C.c_int64, C.c_int64, i64p, u64p)
_sig("orc_tile_bytes", C.c_int64, i64p)
_sig("orc_paged_append", C.c_int, vp, i64p, C.c_int64, C.c_int64, vp, vp, C.c_int64, C.c_int64, C.c_int64,
     i64p, C.c_int64)
_sig("orc_paged_gather", C.c_int, vp, i64p, C.c_int64, i32p, C.c_int64, i32p, C.c_int64, vp, vp)
_sig("orc_paged_gather_mt", C.c_int, vp, i64p, C.c_int64, i32p, C.c_int64, i32p, C.c_int64, vp, vp, C.c_int)
_sig("orc_copy_blocks", C.c_int, vp, i64p, i32p, i32p, C.c_int64)
_sig("orc_paged_append_quant", C.c_int, vp, i64p, C.c_int64, C.c_int64, vp, vp, C.c_int, C.c_int64, C.c_int64,
     C.c_int64, i64p, C.c_int64)
_sig("orc_paged_gather_dequant", C.c_int, vp, i64p, C.c_int64, i32p, C.c_int64, i32p, C.c_int64, vp, vp, C.c_int,
     C.c_int)
_sig("orc_prefix_admit", C.c_int, vp, vp, u32p, i64p, u64p, i64p, C.c_int64, i64p, i64p, C.c_int64, i64p, i64p)
_sig("orc_f32_to_dtype", None, f32p, vp, C.c_int64, C.c_int)
_sig("orc_dtype_to_f32", None, vp, f32p, C.c_int64, C.c_int)

F32, F16, BF16 = 0, 1, 2
ERR = {1: "out of range", 2: "double free", 3: "overflow", 4: "cannot increment ref on free block",
       5: "bad argument"}


class OracleError(RuntimeError):
    def __init__(self, code):
        super().__init__(ERR.get(code, f"error {code}"))
        self.code = code


def _chk(rc):
    if rc:
        raise OracleError(rc)


def _a(x, dt):
    return np.ascontiguousarray(np.asarray(x, dtype=dt))


def _p(a, t):
    return a.ctypes.data_as(t)


class PagedCacheManager:
    """paged_cache.rs:71-302 restated."""

    def __init__(self, block_size, num_blocks):
        self._h = _l.orc_mgr_new(block_size, num_blocks)
        self._bs = block_size

    def __del__(self):
        if getattr(self, "_h", None):
            _l.orc_mgr_delete(self._h)

    def allocate(self) -> Optional[int]:
        o = sz()
        return o.value if _l.orc_mgr_allocate(self._h, C.byref(o)) else None

    def free(self, bid):
        _chk(_l.orc_mgr_free(self._h, bid))

    def ref_count(self, bid):
        o = sz()
        _chk(_l.orc_mgr_ref_count(self._h, bid, C.byref(o)))
        return o.value

    def increment_ref(self, bid):
        _chk(_l.orc_mgr_increment_ref(self._h, bid))

    def copy_on_write(self, bid) -> Optional[int]:
        o, c = sz(), C.c_int()
        _chk(_l.orc_mgr_copy_on_write(self._h, bid, C.byref(o), C.byref(c)))
        return o.value if c.value else None

    def num_free_blocks(self):
        return _l.orc_mgr_num_free(self._h)

    def num_allocated_blocks(self):
        return _l.orc_mgr_num_allocated(self._h)

    def register_hash(self, bid, h):
        _chk(_l.orc_mgr_register_hash(self._h, bid, h))

    def lookup_hash(self, h) -> Optional[int]:
        o = sz()
        return o.value if _l.orc_mgr_lookup_hash(self._h, h, C.byref(o)) else None

    def append_tokens(self, bid, toks):
        a = _a(toks, np.uint32)
        _chk(_l.orc_mgr_append_tokens(self._h, bid, _p(a, u32p), len(a)))

    def get_block(self, bid):
        """(ref_count, hash or None, tokens, num_filled) or None."""
        ref, hh, h, nf, nt = sz(), C.c_int(), C.c_uint64(), sz(), sz()
        toks = (C.c_uint32 * max(self._bs, 1))()
        if not _l.orc_mgr_get_block(self._h, bid, C.byref(ref), C.byref(hh), C.byref(h), C.byref(nf), toks,
                                    self._bs, C.byref(nt)):
            return None
        return ref.value, (h.value if hh.value else None), list(toks[:nt.value]), nf.value


class PrefixCacheManager:
    """prefix_cache.rs:44-292 restated."""

    def __init__(self, max_blocks):
        self._h = _l.orc_prefix_new(max_blocks)
        self.max = max_blocks

    def __del__(self):
        if getattr(self, "_h", None):
            _l.orc_prefix_delete(self._h)

    def lookup(self, toks) -> List[int]:
        a = _a(toks, np.uint32)
        out = np.empty(max(len(a), 1), dtype=np.uint64)
        n = _l.orc_prefix_lookup(self._h, _p(a, u32p), len(a), _p(out, szp), len(out))
        return [int(x) for x in out[:n]]

    def insert(self, toks, ids):
        a, b = _a(toks, np.uint32), _a(ids, np.uint64)
        _l.orc_prefix_insert(self._h, _p(a, u32p), len(a), _p(b, szp), len(b))

    def insert_report(self, toks, ids):
        """insert, returning (attached, replaced) per block."""
        t = _a(toks, np.uint32) if len(toks) else np.zeros(1, np.uint32)
        b = _a(ids, np.uint64).view(np.uintp) if len(ids) else np.zeros(1, np.uintp)
        att = np.zeros(max(len(ids), 1), np.int32)
        rep = np.zeros(max(len(ids), 1), np.int64)
        _l.orc_prefix_insert_report(self._h, _p(t, u32p), len(toks), _p(b, szp), len(ids),
                                    att.ctypes.data_as(C.POINTER(C.c_int32)), _p(rep, i64p))
        return att[:len(ids)], rep[:len(ids)]

    def evict_lru(self) -> Optional[int]:
        o = sz()
        return o.value if _l.orc_prefix_evict_lru(self._h, C.byref(o)) else None

    def hit_rate(self):
        return _l.orc_prefix_hit_rate(self._h)

    def num_blocks(self):
        return _l.orc_prefix_num_blocks(self._h)

    def max_blocks(self):
        return self.max

    def is_full(self):
        return self.num_blocks() >= self.max

    def num_nodes(self):
        return _l.orc_prefix_num_nodes(self._h)


class MemoryAwarePrefixCache:
    """memory.rs:10-200 restated (Linux build)."""

    def __init__(self, max_blocks, memory_limit_mb, bytes_per_block=4096):
        self._h = _l.orc_mem_new(max_blocks, memory_limit_mb, bytes_per_block)

    def __del__(self):
        if getattr(self, "_h", None):
            _l.orc_mem_delete(self._h)

    def insert(self, toks, ids):
        a, b = _a(toks, np.uint32), _a(ids, np.uint64)
        _l.orc_mem_insert(self._h, _p(a, u32p), len(a), _p(b, szp), len(b))

    def lookup(self, toks):
        a = _a(toks, np.uint32)
        out = np.empty(max(len(a), 1), dtype=np.uint64)
        n = _l.orc_mem_lookup(self._h, _p(a, u32p), len(a), _p(out, szp), len(out))
        return [int(x) for x in out[:n]]

    def evict_lru(self):
        o = sz()
        return o.value if _l.orc_mem_evict_lru(self._h, C.byref(o)) else None

    def should_evict(self):
        return bool(_l.orc_mem_should_evict(self._h))

    def current_usage_bytes(self):
        return _l.orc_mem_usage(self._h)

    def memory_limit_bytes(self):
        return _l.orc_mem_limit(self._h)

    def num_blocks(self):
        return _l.orc_mem_num_blocks(self._h)

    def evicted(self) -> List[int]:
        n = _l.orc_mem_evicted(self._h, None, 0)
        out = np.empty(max(n, 1), dtype=np.uint64)
        _l.orc_mem_evicted(self._h, _p(out, szp), n)
        return [int(x) for x in out[:n]]


def quantize_group(data, bits):
    """quantized_cache.rs:232-273 -> (bytes, scale, zero)."""
    d = _a(data, np.float32)
    out = np.zeros(len(d) + 1, dtype=np.uint8)
    s, z = C.c_float(), C.c_float()
    n = _l.orc_quantize_group(_p(d, f32p), len(d), bits, _p(out, u8p), C.byref(s), C.byref(z))
    return out[:n].copy(), np.float32(s.value), np.float32(z.value)


def dequantize_group(b, scale, zero, bits):
    """quantized_cache.rs:278-296."""
    a = _a(b, np.uint8)
    out = np.zeros(2 * len(a) + 1, dtype=np.float32)
    n = _l.orc_dequantize_group(_p(a, u8p), len(a), scale, zero, bits, _p(out, f32p))
    return out[:n].copy()


class QuantizedKVCache:
    """quantized_cache.rs:14-296 restated."""

    def __init__(self, num_layers, num_kv_heads, head_dim, bits, group_size):
        self._h = _l.orc_qcache_new(num_layers, num_kv_heads, head_dim, bits, group_size)
        if not self._h:
            raise OracleError(5)

    def __del__(self):
        if getattr(self, "_h", None):
            _l.orc_qcache_delete(self._h)

    def append(self, layer, keys, values, new_tokens):
        k, v = _a(keys, np.float32), _a(values, np.float32)
        _chk(_l.orc_qcache_append(self._h, layer, _p(k, f32p), _p(v, f32p), len(k), new_tokens))

    def _get(self, layer, which):
        n = sz()
        _l.orc_qcache_get_dequantized(self._h, layer, which, None, 0, C.byref(n))
        out = np.empty(max(n.value, 1), dtype=np.float32)
        _chk(_l.orc_qcache_get_dequantized(self._h, layer, which, _p(out, f32p), len(out), C.byref(n)))
        return out[:n.value]

    def get_keys_dequantized(self, layer):
        return self._get(layer, 0)

    def get_values_dequantized(self, layer):
        return self._get(layer, 1)

    def raw(self, layer, which):
        ng = sz()
        nb = _l.orc_qcache_raw(self._h, layer, which, None, 0, None, None, 0, C.byref(ng))
        b = np.empty(max(nb, 1), dtype=np.uint8)
        s = np.empty(max(ng.value, 1), dtype=np.float32)
        z = np.empty(max(ng.value, 1), dtype=np.float32)
        _l.orc_qcache_raw(self._h, layer, which, _p(b, u8p), nb, _p(s, f32p), _p(z, f32p), ng.value, C.byref(ng))
        return b[:nb], s[:ng.value], z[:ng.value]

    def seq_len(self):
        return _l.orc_qcache_seq_len(self._h)


class RotatingKVCache:
    """rotating_cache.rs:16-283 restated."""

    def __init__(self, num_layers, num_kv_heads, head_dim, max_size, keep):
        self._h = _l.orc_rot_new(num_layers, num_kv_heads, head_dim, max_size, keep)
        if not self._h:
            raise OracleError(5)
        self.heads, self.hd = num_kv_heads, head_dim

    def __del__(self):
        if getattr(self, "_h", None):
            _l.orc_rot_delete(self._h)

    def append(self, layer, keys, values, new_tokens):
        k, v = _a(keys, np.float32), _a(values, np.float32)
        _chk(_l.orc_rot_append(self._h, layer, _p(k, f32p), _p(v, f32p), len(k), new_tokens))

    def seq_len(self):
        return _l.orc_rot_seq_len(self._h)

    def _get(self, layer, vals):
        L = self.seq_len()
        out = np.empty(max(self.heads * L * self.hd, 1), dtype=np.float32)
        _l.orc_rot_get(self._h, layer, vals, _p(out, f32p))
        return [out[h * L * self.hd:(h + 1) * L * self.hd].tolist() for h in range(self.heads)]

    def get_keys(self, layer):
        return self._get(layer, 0)

    def get_values(self, layer):
        return self._get(layer, 1)

    def trim(self, n):
        _chk(_l.orc_rot_trim(self._h, n))


STAT_NAMES = ("requests", "admitted", "rejected", "hit_blocks", "new_blocks", "evictions", "lookup_tokens")


def prefix_admit(mgr: "PagedCacheManager", prefix: "PrefixCacheManager", tokens, cu_tokens, hashes, cu_blocks):
    """Admission policy restated (see kv_oracle.cc): (block_ids, evicted, stats)."""
    t = _a(tokens, np.uint32) if len(tokens) else np.zeros(1, np.uint32)
    cu, cub = _a(cu_tokens, np.int64), _a(cu_blocks, np.int64)
    hs = _a(hashes, np.uint64) if len(hashes) else np.zeros(1, np.uint64)
    nreq = len(cu) - 1
    ids = np.zeros(max(int(cub[-1]), 1), dtype=np.int64)
    cap = int(cub[-1]) * 4 + 16
    ev = np.zeros(cap, dtype=np.int64)
    nev = C.c_int64()
    st = np.zeros(7, dtype=np.int64)
    _chk(_l.orc_prefix_admit(mgr._h, prefix._h, _p(t, u32p), _p(cu, i64p), _p(hs, u64p), _p(cub, i64p), nreq,
                             _p(ids, i64p), _p(ev, i64p), cap, C.byref(nev), _p(st, i64p)))
    return ids[:int(cub[-1])], ev[:min(nev.value, cap)], dict(zip(STAT_NAMES, st.tolist())), nev.value


def xxh64(data: bytes, seed: int = 0) -> int:
    a = np.frombuffer(data, dtype=np.uint8).copy() if data else np.zeros(1, dtype=np.uint8)
    return int(_l.orc_xxh64(_p(a, u8p), len(data), seed))


def hash_chains(tokens, cu_tokens, roots, block_size):
    """Chain hash of every block; returns (hashes, cu_blocks)."""
    t = _a(tokens, np.uint32) if len(tokens) else np.zeros(1, dtype=np.uint32)
    cu = _a(cu_tokens, np.int64)
    r = _a(roots, np.uint64)
    nreq = len(cu) - 1
    nb = (np.diff(cu) + block_size - 1) // block_size
    cub = np.zeros(nreq + 1, dtype=np.int64)
    cub[1:] = np.cumsum(nb)
    out = np.zeros(max(int(cub[-1]), 1), dtype=np.uint64)
    _l.orc_hash_chains(_p(t, u32p), _p(cu, i64p), _p(r, u64p), nreq, block_size, _p(cub, i64p), _p(out, u64p))
    return out[:int(cub[-1])], cub


class Geo:
    """Pool geometry (block-major): layers, heads, head_dim, block_size,
    num_blocks, elem_bytes, bits, group_size, meta_bytes."""

    def __init__(self, layers, heads, head_dim, block_size, num_blocks, elem_bytes=2, bits=0, group_size=64,
                 meta_bytes=4):
        self.v = np.array([layers, heads, head_dim, block_size, num_blocks, elem_bytes, bits, group_size,
                           meta_bytes], dtype=np.int64)
        self.layers, self.heads, self.hd, self.bs, self.nblocks = layers, heads, head_dim, block_size, num_blocks

    @property
    def p(self):
        return _p(self.v, i64p)

    def tile_bytes(self):
        return int(_l.orc_tile_bytes(self.p))

    def pool_bytes(self):
        return self.tile_bytes() * self.layers * 2 * self.heads * self.nblocks


def paged_append(pool: np.ndarray, g: Geo, l0, nl, k: np.ndarray, v: np.ndarray, ls, ts, hs, slots):
    s = _a(slots, np.int64)
    return _l.orc_paged_append(pool.ctypes.data, g.p, l0, nl, k.ctypes.data, v.ctypes.data, ls, ts, hs,
                               _p(s, i64p), len(s))


def paged_gather(pool: np.ndarray, g: Geo, layer, bt: np.ndarray, bt_stride, lens, out_k, out_v, threads=1):
    bt = _a(bt, np.int32)
    ln = _a(lens, np.int32)
    return _l.orc_paged_gather_mt(pool.ctypes.data, g.p, layer, _p(bt, i32p), bt_stride, _p(ln, i32p), len(ln),
                                  out_k.ctypes.data, out_v.ctypes.data, threads)


def copy_blocks(pool: np.ndarray, g: Geo, src, dst):
    a, b = _a(src, np.int32), _a(dst, np.int32)
    return _l.orc_copy_blocks(pool.ctypes.data, g.p, _p(a, i32p), _p(b, i32p), len(a))


def paged_append_quant(pool, g: Geo, l0, nl, k, v, in_dt, ls, ts, hs, slots):
    s = _a(slots, np.int64)
    return _l.orc_paged_append_quant(pool.ctypes.data, g.p, l0, nl, k.ctypes.data, v.ctypes.data, in_dt, ls, ts,
                                     hs, _p(s, i64p), len(s))


def paged_gather_dequant(pool, g: Geo, layer, bt, bt_stride, lens, out_k, out_v, out_dt, threads=1):
    bt = _a(bt, np.int32)
    ln = _a(lens, np.int32)
    return _l.orc_paged_gather_dequant(pool.ctypes.data, g.p, layer, _p(bt, i32p), bt_stride, _p(ln, i32p),
                                       len(ln), out_k.ctypes.data, out_v.ctypes.data, out_dt, threads)


def f32_to_dtype(x: np.ndarray, dt: int) -> np.ndarray:
    """RNE conversion to the storage type, returned as raw uint16/float32."""
    x = _a(x, np.float32)
    out = np.empty(x.shape, dtype=np.float32 if dt == F32 else np.uint16)
    _l.orc_f32_to_dtype(_p(x, f32p), out.ctypes.data, x.size, dt)
    return out


def dtype_to_f32(x: np.ndarray, dt: int) -> np.ndarray:
    x = np.ascontiguousarray(x)
    out = np.empty(x.shape, dtype=np.float32)
    _l.orc_dtype_to_f32(x.ctypes.data, _p(out, f32p), x.size, dt)
    return out
