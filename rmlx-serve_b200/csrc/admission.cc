// Batched prefix-cache admission: the policy that ties PagedCacheManager
// (paged_cache.rs:71-302) and PrefixCacheManager (prefix_cache.rs:44-292)
// together.  The reference never wires the two up -- the scheduler holds a
// PrefixCacheManager that is always None (rmlx-serve-scheduler
// scheduler.rs:168-172) -- so this policy is defined here:
//
// For each request, in order, with n tokens in nb = ceil(n / block_size)
// blocks of which nfull are full, and hashes[b] its chain hashes:
//  1. prefix.lookup(first nfull * block_size tokens): LRU touch and hit stats;
//  2. for every full block b: a block registered under hashes[b] is reused
//     (the request takes a reference) -- blocks are matched one by one, so a
//     block the trie evicted from the middle of a prefix is recomputed while
//     the blocks after it are still reused;
//  3. every other block is allocated; while the pool is empty the LRU block
//     of the prefix cache is evicted and its cache reference dropped; if the
//     cache has nothing left to evict the request is rejected (its
//     references are released, its block ids reported as -1);
//  4. new blocks get their token ids, full ones their hash;
//  5. the full-block prefix is inserted into the prefix cache, which takes a
//     reference on every block it starts holding (at a node that had none,
//     or in place of another block) and drops the one it held on a block it
//     replaces;
//  6. the request releases its own references (prefill-only admission: what
//     stays allocated is exactly what the prefix cache holds).
#include <new>
#include <vector>

#include "block_manager.h"
#include "prefix_cache.h"

using rmlx::fail;

extern "C" rmlx_status rmlx_prefix_admit(rmlx_block_manager* mh, rmlx_prefix_cache* ph, const uint32_t* tokens,
                                         const int64_t* cu_tokens, const uint64_t* hashes, const int64_t* cu_blocks,
                                         int32_t num_requests, int32_t* block_ids, int32_t* evicted,
                                         size_t evicted_cap, size_t* n_evicted, rmlx_admit_stats* stats) {
  if (!mh || !ph || !cu_tokens || !cu_blocks || !block_ids || !n_evicted || !stats)
    return fail(RMLX_E_BAD_ARG, "NULL argument");
  if (num_requests < 0) return fail(RMLX_E_BAD_ARG, "num_requests < 0");
  rmlx::BlockManager& m = mh->impl;
  rmlx::PrefixTrie& p = ph->impl;
  const int64_t bs = (int64_t)m.block_size();
  *stats = rmlx_admit_stats{};
  *n_evicted = 0;
  // Validate the layout before touching any state.
  for (int32_t r = 0; r < num_requests; ++r) {
    const int64_t n = cu_tokens[r + 1] - cu_tokens[r];
    if (n < 0) return fail(RMLX_E_BAD_ARG, "request %d has a negative length", r);
    if (cu_blocks[r + 1] - cu_blocks[r] != (n + bs - 1) / bs)
      return fail(RMLX_E_BAD_ARG, "request %d: cu_blocks does not give ceil(len / block_size) blocks", r);
    if (n > 0 && (!tokens || !hashes)) return fail(RMLX_E_BAD_ARG, "NULL tokens or hashes");
  }
  std::vector<int32_t> scratch;
  std::vector<uint8_t> attached;
  std::vector<int32_t> replaced;
  for (int32_t r = 0; r < num_requests; ++r) {
    const int64_t n = cu_tokens[r + 1] - cu_tokens[r];
    const uint32_t* t = tokens + cu_tokens[r];
    const uint64_t* h = hashes + cu_blocks[r];
    int32_t* ids = block_ids + cu_blocks[r];
    const int64_t nb = cu_blocks[r + 1] - cu_blocks[r];
    const int64_t nfull = n / bs;
    stats->requests += 1;
    stats->lookup_tokens += (size_t)(nfull * bs);
    // 1. LRU touch
    scratch.resize((size_t)(nfull * bs) + 1);
    p.lookup(t, (size_t)(nfull * bs), scratch.data());
    // 2. reuse registered full blocks
    for (int64_t b = 0; b < nb; ++b) {
      ids[b] = -1;
      int32_t id;
      if (b < nfull && m.lookup_hash(h[b], &id)) {
        m.increment_ref(id);
        ids[b] = id;
        stats->hit_blocks += 1;
      }
    }
    // 3. allocate the rest, evicting LRU cache blocks while the pool is empty
    bool rejected = false;
    for (int64_t b = 0; b < nb && !rejected; ++b) {
      if (ids[b] >= 0) continue;
      int32_t id;
      while (!m.allocate(&id)) {
        int32_t victim;
        if (!p.evict_lru(&victim)) {
          rejected = true;
          break;
        }
        m.free_block(victim);
        if (*n_evicted < evicted_cap && evicted) evicted[*n_evicted] = victim;
        *n_evicted += 1;
        stats->evictions += 1;
      }
      if (rejected) break;
      ids[b] = id;
      stats->new_blocks += 1;
      // 4. token ids and, for full blocks, the content hash
      const int64_t cnt = (b + 1) * bs <= n ? bs : n - b * bs;
      m.append_tokens(id, t + b * bs, (size_t)cnt);
      if (b < nfull) m.register_hash(id, h[b]);
    }
    if (rejected) {
      for (int64_t b = 0; b < nb; ++b)
        if (ids[b] >= 0) m.free_block(ids[b]);
      for (int64_t b = 0; b < nb; ++b) ids[b] = -1;
      stats->rejected += 1;
      continue;
    }
    // 5. the prefix cache keeps the full-block prefix
    if (nfull > 0) {
      attached.assign((size_t)nfull, 0);
      replaced.assign((size_t)nfull, -1);
      p.insert_report(t, (size_t)(nfull * bs), ids, (size_t)nfull, attached.data(), replaced.data());
      for (int64_t b = 0; b < nfull; ++b) {
        if (attached[b] || replaced[b] >= 0) m.increment_ref(ids[b]);
        if (replaced[b] >= 0) m.free_block(replaced[b]);
      }
    }
    // 6. release the request's own references
    for (int64_t b = 0; b < nb; ++b) m.free_block(ids[b]);
    stats->admitted += 1;
  }
  return RMLX_OK;
}
