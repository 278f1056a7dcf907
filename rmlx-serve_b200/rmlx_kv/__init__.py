"""rmlx_kv -- B200-native paged KV-cache store for rmlx-serve.

Python mirror of the C ABI in include/rmlx_kv.h, which is the drop-in for
the rmlx-serve-cache crate (crates/rmlx-serve-cache/src/lib.rs:30-40).
"""
from ._lib import BF16, F16, F32, RmlxError, LIB_PATH  # noqa: F401
from .cache import (KVCacheBlock, MemoryAwarePrefixCache, PagedCacheManager,  # noqa: F401
                    PrefixCacheManager, QuantizedKVCache, prefix_admit)
from .pool import KVPool, NcclComm, hash_block_chains  # noqa: F401
from .prompt_cache import (can_trim_prompt_cache, load_prompt_cache, prompt_cache_info,  # noqa: F401
                           read_prompt_cache, save_prompt_cache, trim_prompt_cache, write_prompt_cache)

__all__ = ["KVCacheBlock", "PagedCacheManager", "PrefixCacheManager", "MemoryAwarePrefixCache",
           "QuantizedKVCache", "prefix_admit", "KVPool", "NcclComm", "hash_block_chains",
           "save_prompt_cache", "load_prompt_cache", "prompt_cache_info", "write_prompt_cache", "read_prompt_cache",
           "trim_prompt_cache", "can_trim_prompt_cache", "RmlxError", "F32", "F16", "BF16"]
