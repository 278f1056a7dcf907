/*
 * rmlx_kv.h -- C ABI of the B200 paged KV-cache store.
 *
 * Drop-in for the KV-cache crate of rmlx-serve (crates/rmlx-serve-cache).
 * The reference is a Rust crate with no FFI of its own; every entry point
 * below replaces one public item of that crate (cited as file:line relative
 * to the crate's src/ directory) or is a device operation the crate's types
 * describe but leave to an external GPU library (cited likewise).
 *
 * Conventions
 *   - Every call returns rmlx_status (0 = RMLX_OK).  Where the reference
 *     panics (assert!), the call returns the matching error code and leaves
 *     the state untouched.  Where it returns Option::None, the call returns
 *     RMLX_OK with *found (or *copied) = 0.
 *   - Block ids are int32_t (the reference uses usize); tokens are uint32_t;
 *     hashes are uint64_t; counts are size_t.
 *   - Handles are not thread-safe; the caller serialises calls on one handle,
 *     as the reference's &mut self methods require.
 *   - Device entry points take device pointers and a stream (a cudaStream_t
 *     passed as void*, NULL = the legacy default stream); they enqueue work
 *     and return without synchronising.  Device-side validation failures (a
 *     block id or slot outside the pool) skip the offending row and latch an
 *     error word that rmlx_kv_pool_check() reads back.
 *   - rmlx_last_error() returns a thread-local message for the last failure.
 */
#ifndef RMLX_KV_H
#define RMLX_KV_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RMLX_API __attribute__((visibility("default")))
#else
#define RMLX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum rmlx_status {
  RMLX_OK = 0,
  RMLX_E_RANGE = 1,       /* block id out of range   (paged_cache.rs:126-130) */
  RMLX_E_DOUBLE_FREE = 2, /* free of a free block    (paged_cache.rs:132-135) */
  RMLX_E_OVERFLOW = 3,    /* append past block_size  (paged_cache.rs:290-296) */
  RMLX_E_FREE_BLOCK = 4,  /* share a free block      (paged_cache.rs:177-180) */
  RMLX_E_BAD_ARG = 5,     /* bits/length/layout misuse (quantized_cache.rs:57-60,97-108) */
  RMLX_E_EXHAUSTED = 6,   /* device memory or capacity exhausted */
  RMLX_E_CUDA = 7,        /* a CUDA runtime call failed */
  RMLX_E_NCCL = 8,        /* an NCCL call failed */
  RMLX_E_TIMEOUT = 9,     /* a bounded wait ran out */
  RMLX_E_DEVICE = 10      /* a kernel flagged an out-of-pool block id or slot */
} rmlx_status;

typedef enum rmlx_dtype { RMLX_F32 = 0, RMLX_F16 = 1, RMLX_BF16 = 2 } rmlx_dtype;

RMLX_API const char* rmlx_status_string(rmlx_status s);
RMLX_API const char* rmlx_last_error(void);
/* Library version, e.g. "0.1.0". */
RMLX_API const char* rmlx_version(void);

/* ======================================================================
 * PagedCacheManager -- paged_cache.rs:71-302 (block allocator, refcounts,
 * copy-on-write metadata, content-hash index).  Host-side metadata.
 * ==================================================================== */
typedef struct rmlx_block_manager rmlx_block_manager;

/* KVCacheBlock view -- paged_cache.rs:14-26 */
typedef struct rmlx_block_view {
  int32_t block_id;
  size_t ref_count;
  int32_t has_hash; /* hash: Option<u64> */
  uint64_t hash;
  size_t num_filled;
} rmlx_block_view;

/* PagedCacheManager::new -- paged_cache.rs:90-104 */
RMLX_API rmlx_status rmlx_block_manager_new(size_t block_size, size_t num_blocks, rmlx_block_manager** out);
RMLX_API void rmlx_block_manager_destroy(rmlx_block_manager* m);
/* allocate -- paged_cache.rs:110-115.  *found = 0 when the pool is empty. */
RMLX_API rmlx_status rmlx_block_manager_allocate(rmlx_block_manager* m, int32_t* block_id, int32_t* found);
/* Batched allocate (n calls of allocate in order); *n_got < n when exhausted. */
RMLX_API rmlx_status rmlx_block_manager_allocate_n(rmlx_block_manager* m, size_t n, int32_t* block_ids, size_t* n_got);
/* free -- paged_cache.rs:125-149 */
RMLX_API rmlx_status rmlx_block_manager_free(rmlx_block_manager* m, int32_t block_id);
/* Batched free (n calls of free in order; stops at the first error). */
RMLX_API rmlx_status rmlx_block_manager_free_n(rmlx_block_manager* m, const int32_t* block_ids, size_t n);
/* ref_count -- paged_cache.rs:157-163 */
RMLX_API rmlx_status rmlx_block_manager_ref_count(const rmlx_block_manager* m, int32_t block_id, size_t* out);
/* increment_ref -- paged_cache.rs:172-182 */
RMLX_API rmlx_status rmlx_block_manager_increment_ref(rmlx_block_manager* m, int32_t block_id);
/* copy_on_write -- paged_cache.rs:197-224.  *copied = 0 for None (unshared
 * block, or no free block); the KV bytes are moved by rmlx_kv_copy_blocks. */
RMLX_API rmlx_status rmlx_block_manager_copy_on_write(rmlx_block_manager* m, int32_t block_id, int32_t* new_id,
                                             int32_t* copied);
/* num_free_blocks / num_allocated_blocks / num_blocks / block_size --
 * paged_cache.rs:227-244 */
RMLX_API size_t rmlx_block_manager_num_free_blocks(const rmlx_block_manager* m);
RMLX_API size_t rmlx_block_manager_num_allocated_blocks(const rmlx_block_manager* m);
RMLX_API size_t rmlx_block_manager_num_blocks(const rmlx_block_manager* m);
RMLX_API size_t rmlx_block_manager_block_size(const rmlx_block_manager* m);
/* get_block -- paged_cache.rs:249-251.  *found = 0 when out of range.  Up to
 * `cap` token ids are copied to `tokens` (may be NULL when cap = 0). */
RMLX_API rmlx_status rmlx_block_manager_get_block(const rmlx_block_manager* m, int32_t block_id, rmlx_block_view* view,
                                         uint32_t* tokens, size_t cap, int32_t* found);
/* register_hash -- paged_cache.rs:265-272 */
RMLX_API rmlx_status rmlx_block_manager_register_hash(rmlx_block_manager* m, int32_t block_id, uint64_t hash);
/* lookup_hash -- paged_cache.rs:278-282 */
RMLX_API rmlx_status rmlx_block_manager_lookup_hash(const rmlx_block_manager* m, uint64_t hash, int32_t* block_id,
                                           int32_t* found);
/* append_tokens -- paged_cache.rs:288-301 */
RMLX_API rmlx_status rmlx_block_manager_append_tokens(rmlx_block_manager* m, int32_t block_id, const uint32_t* tokens,
                                             size_t n);

/* ======================================================================
 * PrefixCacheManager -- prefix_cache.rs:44-292 (token trie + LRU).
 * ==================================================================== */
typedef struct rmlx_prefix_cache rmlx_prefix_cache;

/* new -- prefix_cache.rs:66-77 */
RMLX_API rmlx_status rmlx_prefix_cache_new(size_t max_blocks, rmlx_prefix_cache** out);
RMLX_API void rmlx_prefix_cache_destroy(rmlx_prefix_cache* p);
/* lookup -- prefix_cache.rs:85-113.  `block_ids` must hold n entries (a
 * lookup matches at most one block per token); *n_out = matched blocks. */
RMLX_API rmlx_status rmlx_prefix_cache_lookup(rmlx_prefix_cache* p, const uint32_t* tokens, size_t n, int32_t* block_ids,
                                     size_t* n_out);
/* insert -- prefix_cache.rs:126-179 */
RMLX_API rmlx_status rmlx_prefix_cache_insert(rmlx_prefix_cache* p, const uint32_t* tokens, size_t n,
                                     const int32_t* block_ids, size_t n_blocks);
/* evict_lru -- prefix_cache.rs:187-232.  *found = 0 when nothing is cached. */
RMLX_API rmlx_status rmlx_prefix_cache_evict_lru(rmlx_prefix_cache* p, int32_t* block_id, int32_t* found);
/* hit_rate / num_blocks / max_blocks / is_full / num_nodes --
 * prefix_cache.rs:266-291 */
RMLX_API double rmlx_prefix_cache_hit_rate(const rmlx_prefix_cache* p);
RMLX_API size_t rmlx_prefix_cache_num_blocks(const rmlx_prefix_cache* p);
RMLX_API size_t rmlx_prefix_cache_max_blocks(const rmlx_prefix_cache* p);
RMLX_API int32_t rmlx_prefix_cache_is_full(const rmlx_prefix_cache* p);
RMLX_API size_t rmlx_prefix_cache_num_nodes(const rmlx_prefix_cache* p);

/* ======================================================================
 * MemoryAwarePrefixCache -- memory.rs:10-158.  available_memory_mb() is
 * usize::MAX as on the reference's non-macOS build (memory.rs:88-91).
 * ==================================================================== */
typedef struct rmlx_mem_prefix_cache rmlx_mem_prefix_cache;

/* new (bytes_per_block 4096) -- memory.rs:31-45 */
RMLX_API rmlx_status rmlx_mem_prefix_cache_new(size_t max_blocks, size_t memory_limit_mb, rmlx_mem_prefix_cache** out);
/* with_block_size -- memory.rs:53-64 */
RMLX_API rmlx_status rmlx_mem_prefix_cache_with_block_size(size_t max_blocks, size_t memory_limit_mb,
                                                  size_t bytes_per_block, rmlx_mem_prefix_cache** out);
RMLX_API void rmlx_mem_prefix_cache_destroy(rmlx_mem_prefix_cache* p);
/* should_evict -- memory.rs:99-110 */
RMLX_API int32_t rmlx_mem_prefix_cache_should_evict(const rmlx_mem_prefix_cache* p);
/* evict_until_threshold -- memory.rs:117-136 */
RMLX_API rmlx_status rmlx_mem_prefix_cache_evict_until_threshold(rmlx_mem_prefix_cache* p);
/* lookup -- memory.rs:141-143 (same contract as rmlx_prefix_cache_lookup) */
RMLX_API rmlx_status rmlx_mem_prefix_cache_lookup(rmlx_mem_prefix_cache* p, const uint32_t* tokens, size_t n,
                                         int32_t* block_ids, size_t* n_out);
/* insert -- memory.rs:149-158 */
RMLX_API rmlx_status rmlx_mem_prefix_cache_insert(rmlx_mem_prefix_cache* p, const uint32_t* tokens, size_t n,
                                         const int32_t* block_ids, size_t n_blocks);
/* evict_lru -- memory.rs:161-168 */
RMLX_API rmlx_status rmlx_mem_prefix_cache_evict_lru(rmlx_mem_prefix_cache* p, int32_t* block_id, int32_t* found);
/* The reference drops the ids that insert()/evict_until_threshold() evict
 * (memory.rs:121); this pops them, oldest first, so a caller can free the
 * blocks.  *n_out = ids written (<= cap). */
RMLX_API rmlx_status rmlx_mem_prefix_cache_drain_evicted(rmlx_mem_prefix_cache* p, int32_t* block_ids, size_t cap,
                                                size_t* n_out);
RMLX_API double rmlx_mem_prefix_cache_hit_rate(const rmlx_mem_prefix_cache* p);
RMLX_API size_t rmlx_mem_prefix_cache_current_usage_bytes(const rmlx_mem_prefix_cache* p);
RMLX_API size_t rmlx_mem_prefix_cache_memory_limit_bytes(const rmlx_mem_prefix_cache* p);
RMLX_API size_t rmlx_mem_prefix_cache_num_blocks(const rmlx_mem_prefix_cache* p);

/* ======================================================================
 * Prefix-cache admission (host policy glue).  The reference holds a
 * PrefixCacheManager in its scheduler but never sets it (rmlx-serve-
 * scheduler scheduler.rs:168-172); this batched entry admits requests
 * through a PagedCacheManager and a PrefixCacheManager with the policy
 * described in csrc/admission.cc: per-block reuse by chain hash (see
 * rmlx_hash_block_chains), allocation with LRU eviction from the prefix
 * cache while the pool is empty, hash registration of new full blocks,
 * insertion of the full-block prefix (the cache holds one reference per
 * block it holds), then release of the request's own references.
 * ==================================================================== */
typedef struct rmlx_admit_stats {
  size_t requests, admitted, rejected;
  size_t hit_blocks, new_blocks, evictions;
  size_t lookup_tokens;
} rmlx_admit_stats;

/* tokens[cu_tokens[r] .. cu_tokens[r+1]) are request r's token ids and
 * hashes[cu_blocks[r] + b] its chain hashes (host arrays); cu_blocks[r+1] -
 * cu_blocks[r] must be ceil(len / block_size).  On return block_ids[cu_blocks[r]
 * + b] holds the block used for block b (-1 for a rejected request) and
 * evicted[0 .. min(*n_evicted, evicted_cap)) the evicted blocks in order. */
RMLX_API rmlx_status rmlx_prefix_admit(rmlx_block_manager* m, rmlx_prefix_cache* p, const uint32_t* tokens,
                                       const int64_t* cu_tokens, const uint64_t* hashes, const int64_t* cu_blocks,
                                       int32_t num_requests, int32_t* block_ids, int32_t* evicted,
                                       size_t evicted_cap, size_t* n_evicted, rmlx_admit_stats* stats);

/* ======================================================================
 * QuantizedKVCache -- quantized_cache.rs:14-296.  Same host-slice API and
 * byte layout as the reference (per layer, append-call order, groups of
 * group_size over each appended [heads, tokens, head_dim] slice); storage
 * lives in device memory and (de)quantisation runs on the GPU.  Calls are
 * synchronous, like the reference.
 * ==================================================================== */
typedef struct rmlx_qcache rmlx_qcache;

/* new -- quantized_cache.rs:50-81 (bits 4 or 8) */
RMLX_API rmlx_status rmlx_qcache_new(size_t num_layers, size_t num_kv_heads, size_t head_dim, size_t bits,
                            size_t group_size, int device, rmlx_qcache** out);
RMLX_API void rmlx_qcache_destroy(rmlx_qcache* q);
/* append -- quantized_cache.rs:89-127.  keys/values: host f32 slices of
 * length `len` = num_kv_heads * new_tokens * head_dim. */
RMLX_API rmlx_status rmlx_qcache_append(rmlx_qcache* q, size_t layer, const float* keys, const float* values, size_t len,
                               size_t new_tokens);
/* get_keys_dequantized / get_values_dequantized -- quantized_cache.rs:133-151.
 * `out` holds `cap` floats; *n_out = values produced (call with out = NULL,
 * cap = 0 to size the buffer). */
RMLX_API rmlx_status rmlx_qcache_get_keys_dequantized(rmlx_qcache* q, size_t layer, float* out, size_t cap, size_t* n_out);
RMLX_API rmlx_status rmlx_qcache_get_values_dequantized(rmlx_qcache* q, size_t layer, float* out, size_t cap,
                                               size_t* n_out);
/* seq_len / num_layers / bits / group_size -- quantized_cache.rs:154-171 */
RMLX_API size_t rmlx_qcache_seq_len(const rmlx_qcache* q);
RMLX_API size_t rmlx_qcache_num_layers(const rmlx_qcache* q);
RMLX_API size_t rmlx_qcache_bits(const rmlx_qcache* q);
RMLX_API size_t rmlx_qcache_group_size(const rmlx_qcache* q);
/* Stored state of one layer (which = 0 keys, 1 values): packed bytes and the
 * per-group f32 scales and zeros (quantized_cache.rs:16-26).  *n_bytes and
 * *n_groups report the full sizes; up to the caps are copied. */
RMLX_API rmlx_status rmlx_qcache_raw(rmlx_qcache* q, size_t layer, int32_t which, uint8_t* bytes, size_t bytes_cap,
                            float* scales, float* zeros, size_t groups_cap, size_t* n_bytes, size_t* n_groups);

/* Same values as rmlx_qcache_get_keys_dequantized (which = 0) or
 * rmlx_qcache_get_values_dequantized (which = 1), but allocating nothing: the
 * values pass through a fixed device array of RMLX_QCACHE_STATIC_MAX_FLOATS
 * floats (8 MiB) that the library holds on every GPU it is loaded on, until
 * the process exits.  No counterpart in the reference (its cache lives in
 * host memory).  It is for callers that must not call cudaMalloc while they
 * run: an engine that gave nearly all free GPU memory to its KV pool at
 * start-up, where a later allocation can fail or take memory promised to the
 * pool, and per-step code that cannot afford the device-wide synchronisation
 * an allocation may cause.  A layer with more values than the array holds is
 * refused with RMLX_E_BAD_ARG (out = NULL, cap = 0 still reports *n_out).  The
 * first call on a device looks up the array's device address; make that first
 * call before any stream capture.  All calls share the array: calls whose work
 * overlaps on the same GPU race. */
#define RMLX_QCACHE_STATIC_MAX_FLOATS ((size_t)2 * 1024 * 1024)
RMLX_API rmlx_status rmlx_qcache_get_dequantized_static(rmlx_qcache* q, size_t layer, int32_t which, float* out,
                                                        size_t cap, size_t* n_out);

/* ======================================================================
 * Paged KV pool on one GPU (device data plane).
 *
 * The reference keeps KV bytes in rmlx_nn::LayerKvCache, an external GPU
 * buffer per sequence (kv_cache.rs:16-54; appended and read inside the
 * model forward, transformer.rs:125-129).  Its only in-crate value-moving
 * append/gather is RotatingKVCache::append / get_logical_order
 * (rotating_cache.rs:94-197).  The pool below stores those rows in the
 * blocks that PagedCacheManager hands out.
 *
 * Layout (block-major): pool[block][layer][kv][head][slot][row].  One
 * (block, layer, kv, head) tile is block_size rows of head_dim elements
 * (plain pools) or block_size code rows followed by block_size meta rows of
 * head_dim/group_size (scale, zero) pairs (quantised pools), padded to 16 B.
 * A pool holds `num_kv_heads` heads: one KV-head shard of a model when the
 * heads are split over GPUs.
 * ==================================================================== */
typedef struct rmlx_pool_config {
  int32_t num_layers;
  int32_t num_kv_heads; /* heads held by this pool (one shard) */
  int32_t head_dim;
  int32_t block_size;   /* tokens per block (CacheConfig default 16) */
  int32_t num_blocks;
  int32_t dtype;        /* rmlx_dtype of appended and gathered rows */
  int32_t quant_bits;   /* 0 = plain, 8 or 4 = group-affine codes */
  int32_t group_size;   /* quantisation group along head_dim (power of two) */
  int32_t meta_dtype;   /* RMLX_F32 (reference-exact) or RMLX_F16 */
  int32_t head_offset;  /* first global KV head of this shard */
} rmlx_pool_config;

typedef struct rmlx_pool_layout {
  void* base;           /* device pointer of block 0 */
  size_t bytes;         /* total pool bytes */
  size_t tile_bytes;    /* bytes of one (block, layer, kv, head) tile */
  size_t block_bytes;   /* bytes of one block across layers, kv, heads */
  size_t row_bytes;     /* bytes of one stored row (codes for quantised pools) */
  size_t meta_row_bytes;/* bytes of one meta row (0 for plain pools) */
} rmlx_pool_layout;

typedef struct rmlx_kv_pool rmlx_kv_pool;

RMLX_API rmlx_status rmlx_kv_pool_new(const rmlx_pool_config* cfg, int device, rmlx_kv_pool** out);
RMLX_API void rmlx_kv_pool_destroy(rmlx_kv_pool* p);
RMLX_API rmlx_status rmlx_kv_pool_layout(const rmlx_kv_pool* p, rmlx_pool_layout* out);
/* Reads and clears the device error word (synchronises the pool's device). */
RMLX_API rmlx_status rmlx_kv_pool_check(rmlx_kv_pool* p, int32_t* device_error);
/* Copies the device error word into *status on `stream` without waiting for
 * it and without clearing it: the value is valid once the stream has passed
 * this point (an event recorded after it, say).  For a serving loop that
 * reads each step's status without stalling the next step's launches; pass
 * pinned host memory, or the copy is not asynchronous.  No counterpart in
 * the reference crate, whose errors are synchronous panics. */
RMLX_API rmlx_status rmlx_kv_pool_status_async(rmlx_kv_pool* p, int32_t* status, void* stream);

/* Synchronous copies between host memory and pool bytes
 * [offset, offset + nbytes) (raw byte images of the pool; the prompt-cache
 * file format is rmlx_prompt_cache_save / _load below). */
RMLX_API rmlx_status rmlx_kv_pool_read(rmlx_kv_pool* p, size_t offset, size_t nbytes, void* host_dst);
RMLX_API rmlx_status rmlx_kv_pool_write(rmlx_kv_pool* p, size_t offset, size_t nbytes, const void* host_src);

/* Append (reshape-and-cache) -- per-token row copy of
 * RotatingKVCache::append (rotating_cache.rs:126-136) into paged slots.
 * Writes the K and V rows of `num_tokens` tokens for layers
 * [layer_begin, layer_begin + num_layers).  Row (l, t, h) of k/v starts at
 * element (l - layer_begin) * layer_stride + t * token_stride + h * head_stride
 * (element type = cfg.dtype; strides * element size must be multiples of
 * 16 B).  slot_mapping[t] = block * block_size + offset; a negative slot
 * skips the token.  A quantised pool quantises each row on the way in with
 * the group math of quantize_group (quantized_cache.rs:232-273). */
RMLX_API rmlx_status rmlx_kv_append(rmlx_kv_pool* p, int32_t layer_begin, int32_t num_layers, const void* k, const void* v,
                           int64_t layer_stride, int64_t token_stride, int64_t head_stride,
                           const int32_t* slot_mapping, int32_t num_tokens, void* stream);

/* Gather -- RotatingKVCache::get_logical_order (rotating_cache.rs:162-197)
 * over block tables.  For sequence s with length seq_lens[s], writes
 * out[(cu[s] * heads + h * seq_lens[s] + t) * head_dim ...] for every head h
 * and t < seq_lens[s], cu = exclusive prefix sum of seq_lens (sequences
 * packed back to back, each [heads][len][head_dim]).  Row t comes from block
 * block_tables[s * block_table_stride + t / block_size], slot t % block_size.
 * A quantised pool dequantises with the dequantize_group math
 * (quantized_cache.rs:278-296: code * scale + zero, f32, no FMA) and rounds
 * to cfg.dtype.  num_seqs <= RMLX_MAX_SEQS_PER_LAUNCH. */
#define RMLX_MAX_SEQS_PER_LAUNCH 8192
RMLX_API rmlx_status rmlx_kv_gather(rmlx_kv_pool* p, int32_t layer, const int32_t* block_tables, int32_t block_table_stride,
                           const int32_t* seq_lens, int32_t num_seqs, void* out_k, void* out_v, void* stream);

/* Gather of layers [layer_begin, layer_begin + num_layers) in one launch:
 * the same rows as num_layers calls of rmlx_kv_gather, layer layer_begin + i
 * written at out_k / out_v + i * out_layer_stride (elements of cfg.dtype; a
 * multiple of 16 bytes).  The counterpart of rmlx_kv_append's layer range
 * (both replace per-layer get_logical_order calls, rotating_cache.rs:162-197,
 * over a whole step).  One launch walks each pool block's tiles of every
 * layer in pool order and scans seq_lens once; quantised pools are
 * dequantised one launch per layer. */
RMLX_API rmlx_status rmlx_kv_gather_layers(rmlx_kv_pool* p, int32_t layer_begin, int32_t num_layers,
                                           const int32_t* block_tables, int32_t block_table_stride,
                                           const int32_t* seq_lens, int32_t num_seqs, void* out_k, void* out_v,
                                           int64_t out_layer_stride, void* stream);

/* Paged decode attention: the consumer of the K/V tiles, reading them in
 * place (no counterpart in the reference crate, whose attention runs inside
 * the external rmlx-nn layer cache, kv_cache.rs:30,50; listed as the next
 * step after the gather).  For sequence s and query head j of this pool's
 * num_kv_heads x q_heads_per_kv heads (query head j reads KV head
 * j / q_heads_per_kv):
 *   out[s][j][:] = softmax(softmax_scale * q[s][j] . K[s]^T) V[s]
 * over the seq_lens[s] rows that rmlx_kv_gather would return for (s, layer).
 * q and out are [num_seqs][num_kv_heads * q_heads_per_kv][head_dim] in the
 * pool's type; f32 scores and sums; a sequence of length 0 gives zeros.
 * F16/BF16 pools with head_dim 64 or 128, q_heads_per_kv in [1, 16]; a
 * quantised pool (4 or 8 bits) is read as its codes and dequantised in the
 * kernel to the same rows rmlx_kv_gather returns for it.
 * workspace: at least rmlx_kv_attention_workspace_size(...) bytes for a
 * launch whose seq_lens sum to at most max_total_tokens; a launch that needs
 * more is flagged in the pool's device error word (rmlx_kv_pool_check bit 4)
 * and leaves out unwritten.  Launches on one pool hand out work through a
 * counter the pool owns: order them on one stream (or otherwise one after
 * another), not concurrently.  The counter is made with the pool
 * (rmlx_kv_pool_new), so no attention call allocates device memory or
 * synchronises the device. */
RMLX_API rmlx_status rmlx_kv_attention_workspace_size(const rmlx_kv_pool* p, int32_t q_heads_per_kv, int32_t num_seqs,
                                                      int64_t max_total_tokens, size_t* bytes);
RMLX_API rmlx_status rmlx_kv_decode_attention(rmlx_kv_pool* p, int32_t layer, const void* q, int32_t q_heads_per_kv,
                                              const int32_t* block_tables, int32_t block_table_stride,
                                              const int32_t* seq_lens, int32_t num_seqs, float softmax_scale, void* out,
                                              void* workspace, size_t workspace_bytes, void* stream);

/* ---- Batch block tables (the scheduler's KV bookkeeping) -----------------
 * Replaces the per-sequence KVCache / BatchKVCache slots of the scheduler
 * (scheduler.rs:281-436, batch_generator.rs:404-481, 602-630) with block
 * tables over a PagedCacheManager, optionally with a PrefixCacheManager (the
 * scheduler's prefix cache, never set in the reference, scheduler.rs:168-172).
 * No counterpart in the crate itself; the policy is in kv_batch.cc.
 *   add: admits a prompt into the lowest free row; *cached_tokens leading
 *        prompt tokens already sit in reused prefix-cache blocks (prefill may
 *        skip them); slots[0 .. n - cached) are the slots of the rest.
 *        RMLX_E_EXHAUSTED when no row or no block can be had.
 *   step: one token per listed sequence: slots[i] for uids[i]; cow_src/dst
 *        (capacity n) the tiles to copy with rmlx_kv_copy_blocks before the
 *        append.  All-or-nothing: RMLX_E_EXHAUSTED leaves the tables as they
 *        were.
 *   fork / remove (cache_prefix: the finished sequence's full blocks go to
 *        the prefix cache first).
 *   tables: rows [0, *num_rows) as block_tables[row][stride] (0-padded) and
 *        seq_lens[row] (0 for a free row); both NULL = size query.
 * The batch holds references in the block manager: destroy it first.
 * BatchKVCache (batch_cache.rs:13-114) maps onto it as: new(capacity) ->
 * rmlx_kv_batch_new(max_seqs = capacity); insert -> add (the batch picks the
 * lowest free row and returns it); get / get_mut -> seq; remove -> remove;
 * active_count -> num_active; iter -> rows; compact -> nothing to move (a
 * row is a row of the step's block table, a free row a zero-length row that
 * the kernels skip).  KVCache::new / preallocated (kv_cache.rs:28-54) and
 * make_prompt_cache (prompt_cache.rs:31-45) have no per-sequence object: one
 * rmlx_kv_pool_new per GPU holds every sequence's blocks, and add admits a
 * sequence. */
typedef struct rmlx_kv_batch rmlx_kv_batch;
typedef struct {
  uint64_t admitted, rejected, prompt_tokens, cached_tokens, new_blocks, evictions, cow_copies;
} rmlx_batch_stats;
RMLX_API rmlx_status rmlx_kv_batch_new(rmlx_block_manager* m, rmlx_prefix_cache* prefix, int32_t max_seqs,
                                       rmlx_kv_batch** out);
RMLX_API void rmlx_kv_batch_destroy(rmlx_kv_batch* b);
RMLX_API rmlx_status rmlx_kv_batch_add(rmlx_kv_batch* b, uint64_t uid, const uint32_t* prompt, int32_t n, int32_t* row,
                                       int32_t* cached_tokens, int32_t* slots);
RMLX_API rmlx_status rmlx_kv_batch_fork(rmlx_kv_batch* b, uint64_t parent_uid, uint64_t child_uid, int32_t* row);
RMLX_API rmlx_status rmlx_kv_batch_remove(rmlx_kv_batch* b, uint64_t uid, int32_t cache_prefix);
RMLX_API rmlx_status rmlx_kv_batch_step(rmlx_kv_batch* b, const uint64_t* uids, const uint32_t* tokens, int32_t n,
                                        int32_t* slots, int32_t* cow_src, int32_t* cow_dst, int32_t* n_cow);
RMLX_API rmlx_status rmlx_kv_batch_tables(const rmlx_kv_batch* b, int32_t* block_tables, int32_t stride,
                                          int32_t* seq_lens, int32_t max_rows, int32_t* num_rows, int32_t* max_blocks);
RMLX_API rmlx_status rmlx_kv_batch_seq(const rmlx_kv_batch* b, uint64_t uid, int32_t* row, int32_t* len,
                                       int32_t* block_ids, int32_t cap, int32_t* nblocks);
RMLX_API void rmlx_kv_batch_stats(const rmlx_kv_batch* b, rmlx_batch_stats* out);
/* BatchKVCache::active_count (batch_cache.rs:68-70): live sequences. */
RMLX_API int32_t rmlx_kv_batch_num_active(const rmlx_kv_batch* b);
/* BatchKVCache::iter (batch_cache.rs:100-106): for rows [0, min(cap,
 * *num_rows)), uids[row] (0 for a free row) and live[row]; either may be
 * NULL.  *num_rows = max_seqs. */
RMLX_API rmlx_status rmlx_kv_batch_rows(const rmlx_kv_batch* b, uint64_t* uids, int32_t* live, int32_t cap,
                                        int32_t* num_rows);

/* ---- Prompt cache files (prompt_cache.rs:63-210) --------------------------
 * A sequence's K/V as a safetensors file: one [seq_len, head_dim] tensor per
 * (layer, head) named layer_{l}_head_{h}_keys / layer_{l}_head_{h}_values
 * (save_prompt_cache, :55-58), dtype F32/F16/BF16, optional string metadata
 * under "__metadata__", serialised as the safetensors crate does (8-byte LE
 * header length, compact JSON header, tensors ordered by name, header padded
 * to 8 bytes with spaces).  A sequence of length 0 writes no tensors (:79).
 * Heads are named by global index (cfg.head_offset + h).
 *
 * rmlx_prompt_cache_write / _read: host arrays [layers][heads][seq_len]
 * [head_dim] of keys and of values <-> file.  _read takes the heads
 * [head_offset, head_offset + num_kv_heads) of every layer the file holds
 * (the file may hold other heads too) and fails if any is missing; cap_bytes
 * is the size of each of keys and values.
 * rmlx_prompt_cache_info: the file's layers and heads (largest index + 1, as
 * load_prompt_cache derives them, :151-167), seq_len, head_dim, dtype (-1
 * when the file holds no tensor) and its metadata as a JSON object ("" when
 * absent; NUL-terminated, truncated to metadata_cap - 1 bytes).
 * rmlx_prompt_cache_save: the sequence whose rows live in block_ids (host
 * array, block table order) of every layer of the pool -> file (a quantised
 * pool saves its dequantised rows).  rmlx_prompt_cache_load: file -> the
 * rows of the caller-allocated blocks block_ids (ceil(seq_len / block_size)
 * of them; rmlx_prompt_cache_info gives seq_len), through the pool's append;
 * *seq_len = rows loaded.  Both synchronise `stream`. */
RMLX_API rmlx_status rmlx_prompt_cache_write(const char* path, int32_t num_layers, int32_t num_kv_heads, int32_t head_offset,
                                             int32_t seq_len, int32_t head_dim, int32_t dtype, const void* keys,
                                             const void* values, const char* const* meta_keys,
                                             const char* const* meta_values, int32_t num_meta);
RMLX_API rmlx_status rmlx_prompt_cache_read(const char* path, int32_t num_layers, int32_t num_kv_heads, int32_t head_offset,
                                            int32_t head_dim, int32_t dtype, void* keys, void* values, size_t cap_bytes,
                                            int32_t* seq_len);
RMLX_API rmlx_status rmlx_prompt_cache_info(const char* path, int32_t* num_layers, int32_t* num_kv_heads, int32_t* seq_len,
                                            int32_t* head_dim, int32_t* dtype, char* metadata_json, size_t metadata_cap,
                                            size_t* metadata_len);
RMLX_API rmlx_status rmlx_prompt_cache_save(rmlx_kv_pool* p, const int32_t* block_ids, int32_t num_block_ids, int32_t seq_len,
                                            const char* path, const char* const* meta_keys,
                                            const char* const* meta_values, int32_t num_meta, void* stream);
RMLX_API rmlx_status rmlx_prompt_cache_load(rmlx_kv_pool* p, const char* path, const int32_t* block_ids, int32_t num_block_ids,
                                            int32_t* seq_len, void* stream);

/* ---- Rotating (sliding-window) ring over block tables ---------------------
 * RotatingKVCache (rotating_cache.rs:16-283) on paged blocks: a sequence of
 * max_size ring positions keeps its first `keep` and cycles the rest; ring
 * position p is block table entry p / block_size, row p % block_size.  The
 * reference's (written, offset) state lives in an rmlx_rotating (below),
 * which hands out the slot mappings, ring offsets and trim moves for these
 * device calls.
 * rmlx_kv_gather_ring: get_logical_order (:162-197) of layer `layer` for
 * num_seqs sequences: output as rmlx_kv_gather, seq_lens[s] rows; logical
 * row i reads ring position i when ring_offsets[s] < 0 (nothing rotated, the
 * reference's written <= max_size), else i for i < keep and
 * keep + (ring_offsets[s] + i - keep) % (max_size - keep).  Unquantised pools.
 * rmlx_kv_move_rows: row slot src[i] -> slot dst[i] for every layer, K and
 * V and head (codes and scale/zero of a quantised pool), as if all were read
 * before any is written (the shift of trim before rotation, :213-247).
 * src/dst are device arrays; scratch of n rows is allocated on `stream`. */
RMLX_API rmlx_status rmlx_kv_gather_ring(rmlx_kv_pool* p, int32_t layer, const int32_t* block_tables,
                                         int32_t block_table_stride, const int32_t* seq_lens,
                                         const int32_t* ring_offsets, int32_t num_seqs, int32_t keep, int32_t max_size,
                                         void* out_k, void* out_v, void* stream);
RMLX_API rmlx_status rmlx_kv_move_rows(rmlx_kv_pool* p, const int32_t* src_slots, const int32_t* dst_slots, int32_t n,
                                       void* stream);

/* RotatingKVCache's host state (rotating_cache.rs:16-283) for one sequence,
 * over a PagedCacheManager whose blocks hold the ring (destroy the ring
 * before the manager).  The state advances once per token for all of a
 * pool's layers (the reference advances it per per-layer append call: the
 * same for a one-layer cache, or per layer driven as its own cache).
 *   new (:45-83): keep >= max_size -> RMLX_E_BAD_ARG (the reference
 *     panics); block_size must be the manager's.
 *   destroy / release: the ring's blocks go back to the manager (release
 *     keeps the object, empty).
 *   append_slots (:94-143): slots[0..n) of n new tokens, in order, for
 *     rmlx_kv_append; blocks are taken from the manager as the ring first
 *     reaches them, all before any state changes (RMLX_E_EXHAUSTED leaves
 *     the ring unchanged).  A position written twice within one call keeps
 *     the later token; the earlier token's slot is -1 (skipped).
 *   seq_len (:201-203), can_trim (:253-255), written, max_size, keep.
 *   ring_offset: the ring_offsets entry of rmlx_kv_gather_ring: -1 while
 *     written <= max_size, else the reference's offset.
 *   trim (:213-247): n > trimmable -> RMLX_E_RANGE (the reference panics),
 *     state unchanged.  Before the ring rotates, the rows above the trimmed
 *     ones shift down: *n_moves (src, dst) slot pairs for rmlx_kv_move_rows
 *     (at most max_size; RMLX_E_BAD_ARG and no change when cap is short);
 *     after it rotates only the offset moves (*n_moves = 0).
 *   blocks: the ring's block ids in ring order (its block-table row);
 *     *n_blocks always, the ids when out holds them. */
typedef struct rmlx_rotating rmlx_rotating;
RMLX_API rmlx_status rmlx_rotating_new(rmlx_block_manager* m, int32_t block_size, int32_t max_size, int32_t keep,
                                       rmlx_rotating** out);
RMLX_API void rmlx_rotating_destroy(rmlx_rotating* r);
RMLX_API void rmlx_rotating_release(rmlx_rotating* r);
RMLX_API rmlx_status rmlx_rotating_append_slots(rmlx_rotating* r, int32_t n, int32_t* slots);
RMLX_API size_t rmlx_rotating_seq_len(const rmlx_rotating* r);
RMLX_API int32_t rmlx_rotating_can_trim(const rmlx_rotating* r);
RMLX_API int32_t rmlx_rotating_ring_offset(const rmlx_rotating* r);
RMLX_API size_t rmlx_rotating_written(const rmlx_rotating* r);
RMLX_API size_t rmlx_rotating_max_size(const rmlx_rotating* r);
RMLX_API size_t rmlx_rotating_keep(const rmlx_rotating* r);
RMLX_API rmlx_status rmlx_rotating_trim(rmlx_rotating* r, int32_t n, int32_t* src_slots, int32_t* dst_slots,
                                        int32_t cap, int32_t* n_moves);
RMLX_API rmlx_status rmlx_rotating_blocks(const rmlx_rotating* r, int32_t* out, int32_t cap, int32_t* n_blocks);

/* Block copy for copy-on-write / fork: every tile of block src[i] is copied
 * to block dst[i] (all layers, K and V, all heads of the pool).  src/dst are
 * device arrays of n ids; the dst set must not intersect the src set.  This
 * moves the bytes that PagedCacheManager::copy_on_write (paged_cache.rs:
 * 197-224) leaves to the GPU-side cache. */
RMLX_API rmlx_status rmlx_kv_copy_blocks(rmlx_kv_pool* p, const int32_t* src, const int32_t* dst, int32_t n, void* stream);

/* Pack blocks ids[0..n) into a contiguous device staging buffer of
 * n * block_bytes (block-major), and the inverse.  Used for cross-GPU block
 * migration over NCCL. */
RMLX_API rmlx_status rmlx_kv_pack_blocks(rmlx_kv_pool* p, const int32_t* ids, int32_t n, void* staging, void* stream);
RMLX_API rmlx_status rmlx_kv_unpack_blocks(rmlx_kv_pool* p, const int32_t* ids, int32_t n, const void* staging,
                                  void* stream);

/* ======================================================================
 * Prefix-block chain hash (device).  The reference accepts caller-supplied
 * block hashes (PagedCacheManager::register_hash, paged_cache.rs:265-272)
 * and computes none; this defines them.  For request r with tokens
 * tokens[cu_tokens[r] .. cu_tokens[r+1]), block b covers tokens
 * [b*block_size, min((b+1)*block_size, n)) and
 *   hash[b] = XXH64(le64(hash[b-1]) || le32(tokens of block b), seed 0),
 * hash[-1] = root_hashes[r].  Hashes go to out[cu_blocks[r] + b] with
 * cu_blocks[r+1] - cu_blocks[r] = ceil(n / block_size).  All arrays are
 * device arrays. */
RMLX_API rmlx_status rmlx_hash_block_chains(const uint32_t* tokens, const int64_t* cu_tokens, const uint64_t* root_hashes,
                                   int32_t num_requests, int32_t block_size, const int64_t* cu_blocks,
                                   uint64_t* out, void* stream);

/* ======================================================================
 * Cross-GPU block migration (NCCL over NVLink / NVSwitch).  The reference's
 * only multi-device hook is the never-enabled "distributed" feature of
 * rmlx-serve-engine (crates/rmlx-serve-engine/Cargo.toml:24-30); with the pool
 * sharded by KV head, moving blocks between pools on different GPUs is the
 * one exchange: pack -> grouped ncclSend/ncclRecv -> unpack on one stream.
 * Communicators are non-blocking; every wait is bounded by timeout_ms, after
 * which the communicator is aborted and RMLX_E_TIMEOUT is returned.
 * ==================================================================== */
typedef struct rmlx_comm rmlx_comm;
#define RMLX_NCCL_ID_BYTES 128

/* 128-byte NCCL unique id, made on one rank and shared with the others. */
RMLX_API rmlx_status rmlx_nccl_unique_id(uint8_t* out);
/* Communicator of `nranks` processes; this one is `rank`, on `device`. */
RMLX_API rmlx_status rmlx_nccl_comm_new(int32_t nranks, const uint8_t* id, int32_t rank, int device,
                                        int32_t timeout_ms, rmlx_comm** out);
RMLX_API void rmlx_nccl_comm_destroy(rmlx_comm* c);
/* Exchange blocks with `peer` (both ranks call it): send blocks send_ids
 * (device array, n_send) of this pool, receive n_recv blocks into recv_ids.
 * Staging buffers are device buffers of n * block_bytes.  Enqueued on
 * `stream`; rmlx_nccl_wait bounds the completion.
 * Call it only after both ranks have agreed on the counts on the host, each
 * confirming that it can hold what comes, with bounded waits (the Python
 * side's rmlx_kv.distributed.exchange_migration_plan does this through the
 * process group's key-value store): a rank whose peer has left or failed
 * must learn it there, not from a transfer posted toward that peer. */
RMLX_API rmlx_status rmlx_kv_migrate(rmlx_kv_pool* p, rmlx_comm* c, int32_t peer, const int32_t* send_ids,
                                     int32_t n_send, void* send_staging, const int32_t* recv_ids, int32_t n_recv,
                                     void* recv_staging, void* stream);
/* Wait for `stream` (timeout_ms <= 0: the communicator's timeout); on an
 * NCCL error or the deadline the communicator is aborted. */
RMLX_API rmlx_status rmlx_nccl_wait(rmlx_comm* c, void* stream, int32_t timeout_ms);

#ifdef __cplusplus
}
#endif
#endif /* RMLX_KV_H */
