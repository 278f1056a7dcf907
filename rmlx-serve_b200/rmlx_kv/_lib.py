"""ctypes binding of librmlx_kv.so (the C ABI declared in include/rmlx_kv.h).

The shared library is built in-tree (``make -C rmlx-serve_b200``) into
``rmlx-serve_b200/lib/librmlx_kv.so``.  There is no fallback: importing this
module raises if the library is missing.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "librmlx_kv.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `make -C rmlx-serve_b200` "
        "(the KV store has no CPU fallback)")

lib = C.CDLL(LIB_PATH)

# status codes (rmlx_status)
OK, E_RANGE, E_DOUBLE_FREE, E_OVERFLOW, E_FREE_BLOCK, E_BAD_ARG, E_EXHAUSTED, \
    E_CUDA, E_NCCL, E_TIMEOUT, E_DEVICE = range(11)
F32, F16, BF16 = 0, 1, 2


# rmlx_status values (include/rmlx_kv.h)
RMLX_OK, RMLX_E_RANGE, RMLX_E_DOUBLE_FREE, RMLX_E_OVERFLOW, RMLX_E_FREE_BLOCK, RMLX_E_BAD_ARG = 0, 1, 2, 3, 4, 5
RMLX_E_EXHAUSTED, RMLX_E_CUDA, RMLX_E_NCCL, RMLX_E_TIMEOUT, RMLX_E_DEVICE = 6, 7, 8, 9, 10


class RmlxError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{msg} [{lib.rmlx_status_string(status).decode()}]")
        self.status = status


def check(status: int) -> None:
    if status != OK:
        raise RmlxError(status, lib.rmlx_last_error().decode())


c_size_p = C.POINTER(C.c_size_t)
i32p = C.POINTER(C.c_int32)
u32p = C.POINTER(C.c_uint32)
u64p = C.POINTER(C.c_uint64)
i64p = C.POINTER(C.c_int64)
f32p = C.POINTER(C.c_float)
u8p = C.POINTER(C.c_uint8)
vp = C.c_void_p


class BlockView(C.Structure):
    _fields_ = [("block_id", C.c_int32), ("ref_count", C.c_size_t), ("has_hash", C.c_int32),
                ("hash", C.c_uint64), ("num_filled", C.c_size_t)]


class AdmitStats(C.Structure):
    _fields_ = [(n, C.c_size_t) for n in (
        "requests", "admitted", "rejected", "hit_blocks", "new_blocks", "evictions", "lookup_tokens")]


class PoolConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "num_layers", "num_kv_heads", "head_dim", "block_size", "num_blocks", "dtype",
        "quant_bits", "group_size", "meta_dtype", "head_offset")]


class PoolLayout(C.Structure):
    _fields_ = [("base", vp), ("bytes", C.c_size_t), ("tile_bytes", C.c_size_t),
                ("block_bytes", C.c_size_t), ("row_bytes", C.c_size_t),
                ("meta_row_bytes", C.c_size_t)]


def _sig(name, res, *args):
    f = getattr(lib, name)
    f.restype = res
    f.argtypes = list(args)


st = C.c_int
_sig("rmlx_status_string", C.c_char_p, st)
_sig("rmlx_last_error", C.c_char_p)
_sig("rmlx_version", C.c_char_p)

# PagedCacheManager
_sig("rmlx_block_manager_new", st, C.c_size_t, C.c_size_t, C.POINTER(vp))
_sig("rmlx_block_manager_destroy", None, vp)
_sig("rmlx_block_manager_allocate", st, vp, i32p, i32p)
_sig("rmlx_block_manager_allocate_n", st, vp, C.c_size_t, i32p, c_size_p)
_sig("rmlx_block_manager_free", st, vp, C.c_int32)
_sig("rmlx_block_manager_free_n", st, vp, i32p, C.c_size_t)
_sig("rmlx_block_manager_ref_count", st, vp, C.c_int32, c_size_p)
_sig("rmlx_block_manager_increment_ref", st, vp, C.c_int32)
_sig("rmlx_block_manager_copy_on_write", st, vp, C.c_int32, i32p, i32p)
for _n in ("num_free_blocks", "num_allocated_blocks", "num_blocks", "block_size"):
    _sig(f"rmlx_block_manager_{_n}", C.c_size_t, vp)
_sig("rmlx_block_manager_get_block", st, vp, C.c_int32, C.POINTER(BlockView), u32p, C.c_size_t, i32p)
_sig("rmlx_block_manager_register_hash", st, vp, C.c_int32, C.c_uint64)
_sig("rmlx_block_manager_lookup_hash", st, vp, C.c_uint64, i32p, i32p)
_sig("rmlx_block_manager_append_tokens", st, vp, C.c_int32, u32p, C.c_size_t)

# PrefixCacheManager
_sig("rmlx_prefix_cache_new", st, C.c_size_t, C.POINTER(vp))
_sig("rmlx_prefix_cache_destroy", None, vp)
_sig("rmlx_prefix_cache_lookup", st, vp, u32p, C.c_size_t, i32p, c_size_p)
_sig("rmlx_prefix_cache_insert", st, vp, u32p, C.c_size_t, i32p, C.c_size_t)
_sig("rmlx_prefix_cache_evict_lru", st, vp, i32p, i32p)
_sig("rmlx_prefix_cache_hit_rate", C.c_double, vp)
_sig("rmlx_prefix_cache_num_blocks", C.c_size_t, vp)
_sig("rmlx_prefix_cache_max_blocks", C.c_size_t, vp)
_sig("rmlx_prefix_cache_is_full", C.c_int32, vp)
_sig("rmlx_prefix_cache_num_nodes", C.c_size_t, vp)

# MemoryAwarePrefixCache
_sig("rmlx_mem_prefix_cache_new", st, C.c_size_t, C.c_size_t, C.POINTER(vp))
_sig("rmlx_mem_prefix_cache_with_block_size", st, C.c_size_t, C.c_size_t, C.c_size_t, C.POINTER(vp))
_sig("rmlx_mem_prefix_cache_destroy", None, vp)
_sig("rmlx_mem_prefix_cache_should_evict", C.c_int32, vp)
_sig("rmlx_mem_prefix_cache_evict_until_threshold", st, vp)
_sig("rmlx_mem_prefix_cache_lookup", st, vp, u32p, C.c_size_t, i32p, c_size_p)
_sig("rmlx_mem_prefix_cache_insert", st, vp, u32p, C.c_size_t, i32p, C.c_size_t)
_sig("rmlx_mem_prefix_cache_evict_lru", st, vp, i32p, i32p)
_sig("rmlx_mem_prefix_cache_drain_evicted", st, vp, i32p, C.c_size_t, c_size_p)
_sig("rmlx_mem_prefix_cache_hit_rate", C.c_double, vp)
_sig("rmlx_mem_prefix_cache_current_usage_bytes", C.c_size_t, vp)
_sig("rmlx_mem_prefix_cache_memory_limit_bytes", C.c_size_t, vp)
_sig("rmlx_mem_prefix_cache_num_blocks", C.c_size_t, vp)

# admission
_sig("rmlx_prefix_admit", st, vp, vp, u32p, i64p, u64p, i64p, C.c_int32, i32p, i32p, C.c_size_t, c_size_p,
     C.POINTER(AdmitStats))

# QuantizedKVCache
_sig("rmlx_qcache_new", st, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int,
     C.POINTER(vp))
_sig("rmlx_qcache_destroy", None, vp)
_sig("rmlx_qcache_append", st, vp, C.c_size_t, f32p, f32p, C.c_size_t, C.c_size_t)
_sig("rmlx_qcache_get_keys_dequantized", st, vp, C.c_size_t, f32p, C.c_size_t, c_size_p)
_sig("rmlx_qcache_get_values_dequantized", st, vp, C.c_size_t, f32p, C.c_size_t, c_size_p)
for _n in ("seq_len", "num_layers", "bits", "group_size"):
    _sig(f"rmlx_qcache_{_n}", C.c_size_t, vp)
_sig("rmlx_qcache_raw", st, vp, C.c_size_t, C.c_int32, u8p, C.c_size_t, f32p, f32p, C.c_size_t,
     c_size_p, c_size_p)

# device pool
_sig("rmlx_kv_pool_new", st, C.POINTER(PoolConfig), C.c_int, C.POINTER(vp))
_sig("rmlx_kv_pool_destroy", None, vp)
_sig("rmlx_kv_pool_layout", st, vp, C.POINTER(PoolLayout))
_sig("rmlx_kv_pool_check", st, vp, i32p)
_sig("rmlx_kv_pool_status_async", st, vp, vp, vp)
_sig("rmlx_kv_pool_read", st, vp, C.c_size_t, C.c_size_t, vp)
_sig("rmlx_kv_pool_write", st, vp, C.c_size_t, C.c_size_t, vp)
_sig("rmlx_kv_append", st, vp, C.c_int32, C.c_int32, vp, vp, C.c_int64, C.c_int64, C.c_int64, vp,
     C.c_int32, vp)
_sig("rmlx_kv_gather", st, vp, C.c_int32, vp, C.c_int32, vp, C.c_int32, vp, vp, vp)
_sig("rmlx_kv_gather_layers", st, vp, C.c_int32, C.c_int32, vp, C.c_int32, vp, C.c_int32, vp, vp, C.c_int64, vp)
_sig("rmlx_kv_attention_workspace_size", st, vp, C.c_int32, C.c_int32, C.c_int64, C.POINTER(C.c_size_t))
_sig("rmlx_kv_decode_attention", st, vp, C.c_int32, vp, C.c_int32, vp, C.c_int32, vp, C.c_int32, C.c_float, vp, vp,
     C.c_size_t, vp)
_sig("rmlx_kv_copy_blocks", st, vp, vp, vp, C.c_int32, vp)

# RotatingKVCache state over a block manager
_sig("rmlx_rotating_new", st, vp, C.c_int32, C.c_int32, C.c_int32, C.POINTER(vp))
_sig("rmlx_rotating_destroy", None, vp)
_sig("rmlx_rotating_release", None, vp)
_sig("rmlx_rotating_append_slots", st, vp, C.c_int32, i32p)
for _n in ("seq_len", "written", "max_size", "keep"):
    _sig(f"rmlx_rotating_{_n}", C.c_size_t, vp)
_sig("rmlx_rotating_can_trim", C.c_int32, vp)
_sig("rmlx_rotating_ring_offset", C.c_int32, vp)
_sig("rmlx_rotating_trim", st, vp, C.c_int32, i32p, i32p, C.c_int32, i32p)
_sig("rmlx_rotating_blocks", st, vp, i32p, C.c_int32, i32p)


class BatchStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("admitted", "rejected", "prompt_tokens", "cached_tokens", "new_blocks",
                                          "evictions", "cow_copies")]


u64p = C.POINTER(C.c_uint64)
_sig("rmlx_kv_batch_new", st, vp, vp, C.c_int32, C.POINTER(vp))
_sig("rmlx_kv_batch_destroy", None, vp)
_sig("rmlx_kv_batch_add", st, vp, C.c_uint64, u32p, C.c_int32, i32p, i32p, i32p)
_sig("rmlx_kv_batch_fork", st, vp, C.c_uint64, C.c_uint64, i32p)
_sig("rmlx_kv_batch_remove", st, vp, C.c_uint64, C.c_int32)
_sig("rmlx_kv_batch_step", st, vp, u64p, u32p, C.c_int32, i32p, i32p, i32p, i32p)
_sig("rmlx_kv_batch_tables", st, vp, i32p, C.c_int32, i32p, C.c_int32, i32p, i32p)
_sig("rmlx_kv_batch_seq", st, vp, C.c_uint64, i32p, i32p, i32p, C.c_int32, i32p)
_sig("rmlx_kv_batch_stats", None, vp, C.POINTER(BatchStats))
_sig("rmlx_kv_batch_num_active", C.c_int32, vp)
_sig("rmlx_kv_batch_rows", st, vp, u64p, i32p, C.c_int32, i32p)
_sig("rmlx_kv_gather_ring", st, vp, C.c_int32, vp, C.c_int32, vp, vp, C.c_int32, C.c_int32, C.c_int32, vp, vp, vp)
_sig("rmlx_kv_move_rows", st, vp, vp, vp, C.c_int32, vp)
cpp = C.POINTER(C.c_char_p)
_sig("rmlx_prompt_cache_write", st, C.c_char_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, vp,
     vp, cpp, cpp, C.c_int32)
_sig("rmlx_prompt_cache_read", st, C.c_char_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, vp, vp, C.c_size_t,
     C.POINTER(C.c_int32))
_sig("rmlx_prompt_cache_info", st, C.c_char_p, C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_int32),
     C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t))
_sig("rmlx_prompt_cache_save", st, vp, i32p, C.c_int32, C.c_int32, C.c_char_p, cpp, cpp, C.c_int32, vp)
_sig("rmlx_prompt_cache_load", st, vp, C.c_char_p, i32p, C.c_int32, C.POINTER(C.c_int32), vp)
_sig("rmlx_kv_pack_blocks", st, vp, vp, C.c_int32, vp, vp)
_sig("rmlx_kv_unpack_blocks", st, vp, vp, C.c_int32, vp, vp)
_sig("rmlx_hash_block_chains", st, vp, vp, vp, C.c_int32, C.c_int32, vp, vp, vp)

# NCCL migration
_sig("rmlx_nccl_unique_id", st, u8p)
_sig("rmlx_nccl_comm_new", st, C.c_int32, u8p, C.c_int32, C.c_int, C.c_int32, C.POINTER(vp))
_sig("rmlx_nccl_comm_destroy", None, vp)
_sig("rmlx_kv_migrate", st, vp, vp, C.c_int32, vp, C.c_int32, vp, vp, C.c_int32, vp, vp)
_sig("rmlx_nccl_wait", st, vp, vp, C.c_int32)
