// Host-side prefix cache: the drop-in for PrefixCacheManager
// (crates/rmlx-serve-cache/src/prefix_cache.rs:44-292) and
// MemoryAwarePrefixCache (crates/rmlx-serve-cache/src/memory.rs:10-200).
//
// Observable behaviour is the reference's, including its eviction order:
// among nodes holding a block, leaves (no children) before internal nodes,
// then the smallest last_access, ties to the lowest arena index
// (prefix_cache.rs:195-215); every node touched by one lookup/insert gets
// the same access stamp (:92-99, :137-154); nodes are never removed from
// the arena, a pruned leaf is only unlinked from its parent (:235-260).
//
// The data structures differ so that the cost no longer grows with the trie:
//   * children of all nodes live in one open-addressing map keyed by
//     (parent index << 32 | token id) instead of one HashMap per node;
//   * each node records its parent and incoming token, so unlinking a leaf
//     is O(1) rather than a scan of every node's children (:245-259);
//   * nodes that hold a block are kept in an ordered set keyed by
//     (is_internal, last_access, index), so evict_lru is O(log n) instead of
//     a scan of the arena (:199-215) and picks the same victim.
#include <new>

#include "prefix_cache.h"


using rmlx::fail;


extern "C" {

rmlx_status rmlx_prefix_cache_new(size_t max_blocks, rmlx_prefix_cache** out) {
  if (!out) return fail(RMLX_E_BAD_ARG, "out is NULL");
  *out = new (std::nothrow) rmlx_prefix_cache(max_blocks);
  return *out ? RMLX_OK : fail(RMLX_E_EXHAUSTED, "host allocation failed");
}
void rmlx_prefix_cache_destroy(rmlx_prefix_cache* p) { delete p; }
rmlx_status rmlx_prefix_cache_lookup(rmlx_prefix_cache* p, const uint32_t* t, size_t n, int32_t* ids,
                                     size_t* n_out) {
  if (n && (!t || !ids)) return fail(RMLX_E_BAD_ARG, "NULL tokens or block_ids");
  *n_out = p->impl.lookup(t, n, ids);
  return RMLX_OK;
}
rmlx_status rmlx_prefix_cache_insert(rmlx_prefix_cache* p, const uint32_t* t, size_t n, const int32_t* ids,
                                     size_t nb) {
  if ((n && !t) || (nb && !ids)) return fail(RMLX_E_BAD_ARG, "NULL tokens or block_ids");
  p->impl.insert(t, n, ids, nb);
  return RMLX_OK;
}
rmlx_status rmlx_prefix_cache_evict_lru(rmlx_prefix_cache* p, int32_t* id, int32_t* found) {
  *found = p->impl.evict_lru(id) ? 1 : 0;
  return RMLX_OK;
}
double rmlx_prefix_cache_hit_rate(const rmlx_prefix_cache* p) { return p->impl.hit_rate(); }
size_t rmlx_prefix_cache_num_blocks(const rmlx_prefix_cache* p) { return p->impl.num_blocks(); }
size_t rmlx_prefix_cache_max_blocks(const rmlx_prefix_cache* p) { return p->impl.max_blocks(); }
int32_t rmlx_prefix_cache_is_full(const rmlx_prefix_cache* p) { return p->impl.is_full() ? 1 : 0; }
size_t rmlx_prefix_cache_num_nodes(const rmlx_prefix_cache* p) { return p->impl.num_nodes(); }

rmlx_status rmlx_mem_prefix_cache_new(size_t max_blocks, size_t mb, rmlx_mem_prefix_cache** out) {
  return rmlx_mem_prefix_cache_with_block_size(max_blocks, mb, 4096, out);  // memory.rs:37
}
rmlx_status rmlx_mem_prefix_cache_with_block_size(size_t max_blocks, size_t mb, size_t bpb,
                                                  rmlx_mem_prefix_cache** out) {
  if (!out) return fail(RMLX_E_BAD_ARG, "out is NULL");
  *out = new (std::nothrow) rmlx_mem_prefix_cache(max_blocks, mb, bpb);
  return *out ? RMLX_OK : fail(RMLX_E_EXHAUSTED, "host allocation failed");
}
void rmlx_mem_prefix_cache_destroy(rmlx_mem_prefix_cache* p) { delete p; }
int32_t rmlx_mem_prefix_cache_should_evict(const rmlx_mem_prefix_cache* p) { return p->impl.should_evict() ? 1 : 0; }
rmlx_status rmlx_mem_prefix_cache_evict_until_threshold(rmlx_mem_prefix_cache* p) {
  p->impl.evict_until_threshold();
  return RMLX_OK;
}
rmlx_status rmlx_mem_prefix_cache_lookup(rmlx_mem_prefix_cache* p, const uint32_t* t, size_t n, int32_t* ids,
                                         size_t* n_out) {
  if (n && (!t || !ids)) return fail(RMLX_E_BAD_ARG, "NULL tokens or block_ids");
  *n_out = p->impl.trie_.lookup(t, n, ids);
  return RMLX_OK;
}
rmlx_status rmlx_mem_prefix_cache_insert(rmlx_mem_prefix_cache* p, const uint32_t* t, size_t n, const int32_t* ids,
                                         size_t nb) {
  if ((n && !t) || (nb && !ids)) return fail(RMLX_E_BAD_ARG, "NULL tokens or block_ids");
  p->impl.insert(t, n, ids, nb);
  return RMLX_OK;
}
rmlx_status rmlx_mem_prefix_cache_evict_lru(rmlx_mem_prefix_cache* p, int32_t* id, int32_t* found) {
  *found = p->impl.evict_lru(id) ? 1 : 0;
  return RMLX_OK;
}
rmlx_status rmlx_mem_prefix_cache_drain_evicted(rmlx_mem_prefix_cache* p, int32_t* ids, size_t cap,
                                                size_t* n_out) {
  *n_out = p->impl.drain(ids, cap);
  return RMLX_OK;
}
double rmlx_mem_prefix_cache_hit_rate(const rmlx_mem_prefix_cache* p) { return p->impl.trie_.hit_rate(); }
size_t rmlx_mem_prefix_cache_current_usage_bytes(const rmlx_mem_prefix_cache* p) { return p->impl.usage_; }
size_t rmlx_mem_prefix_cache_memory_limit_bytes(const rmlx_mem_prefix_cache* p) { return p->impl.limit_; }
size_t rmlx_mem_prefix_cache_num_blocks(const rmlx_mem_prefix_cache* p) { return p->impl.trie_.num_blocks(); }

}  // extern "C"
