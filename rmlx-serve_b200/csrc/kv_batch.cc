// Block tables of a running batch: the KV bookkeeping of the scheduler's
// admit / step / finish cycle (rmlx-serve-scheduler scheduler.rs:281-436,
// batch_generator.rs:404-481 and find_cache_slot_for_uid :602-630), on the
// paged pool instead of one contiguous KVCache per sequence.  Sequences sit
// in rows 0..max_seqs-1 (the lowest free row is taken, as the reference's
// BatchKVCache slot); one step is one batched append for every listed
// sequence.  A PrefixCacheManager, which the reference's scheduler holds but
// never sets (scheduler.rs:168-172), is used when one is given.
//
// Policy (build-defined; restated in the tests):
//  add(uid, prompt):  prompt's full blocks get chain hashes (chain_hash.h,
//    root 0).  With a prefix cache: lookup (LRU touch, hit statistics), then
//    the leading full blocks whose hash is registered are reused (one
//    reference each) while they match -- at most (n - 1) / block_size of
//    them, so the prompt's last token is always computed -- and those tokens
//    are reported as cached.  The other blocks are allocated in order; while
//    the pool is empty the prefix cache's LRU block is evicted (its cache
//    reference dropped); with nothing left to evict the request is rejected
//    (RMLX_E_EXHAUSTED, its references released).  New blocks get their
//    token ids and, when full, their hash.  The prompt's full-block prefix
//    goes into the prefix cache, which holds one reference on every block it
//    holds.  Slots are returned for the uncached tokens.
//  step(uids, tokens): one token per listed sequence, in order.  A sequence
//    whose next token starts a block needs a new block; one whose last
//    block is shared needs a private copy (the metadata side of
//    copy_on_write, paged_cache.rs:197-224; the caller copies the tile with
//    rmlx_kv_copy_blocks before the append) -- except the block's last
//    holder in the step: once the copies planned before it are made it holds
//    the block alone and writes in place.  All the
//    blocks the step needs are allocated first, in sequence order, evicting
//    as in add; if they cannot all be had, none is kept and the step fails
//    with RMLX_E_EXHAUSTED (evictions done stay done).  A block that fills
//    up gets its chain hash registered.
//  fork(parent, child): the child shares every block of the parent.
//  remove(uid, cache_prefix): with cache_prefix and a prefix cache, the
//    sequence's full-block prefix (prompt and generated tokens) is inserted
//    first; then the sequence's references are released.
#include <algorithm>
#include <new>
#include <unordered_map>
#include <vector>

#include "block_manager.h"
#include "chain_hash.h"
#include "prefix_cache.h"

using rmlx::fail;

namespace {

struct Row {
  bool live = false;
  uint64_t uid = 0;
  std::vector<int32_t> blocks;
  std::vector<uint32_t> tokens;  // every token of the sequence
  std::vector<uint64_t> hashes;  // chain hash of each full block
};

}  // namespace

struct rmlx_kv_batch {
  rmlx::BlockManager* m;
  rmlx::PrefixTrie* p;  // may be null
  std::vector<Row> rows;
  std::unordered_map<uint64_t, int32_t> by_uid;
  rmlx_batch_stats stats{};

  int64_t bs() const { return (int64_t)m->block_size(); }

  // One block, evicting LRU prefix-cache blocks while the pool is empty.
  bool take_block(int32_t* id) {
    while (!m->allocate(id)) {
      int32_t victim;
      if (!p || !p->evict_lru(&victim)) return false;
      m->free_block(victim);
      stats.evictions += 1;
    }
    stats.new_blocks += 1;
    return true;
  }

  // The prefix cache takes the full-block prefix of `t` held in `ids`.
  void cache_prefix(const uint32_t* t, int64_t nfull, const int32_t* ids) {
    if (!p || nfull <= 0) return;
    std::vector<uint8_t> attached((size_t)nfull);
    std::vector<int32_t> replaced((size_t)nfull);
    p->insert_report(t, (size_t)(nfull * bs()), ids, (size_t)nfull, attached.data(), replaced.data());
    for (int64_t b = 0; b < nfull; ++b) {
      if (attached[b] || replaced[b] >= 0) m->increment_ref(ids[b]);
      if (replaced[b] >= 0) m->free_block(replaced[b]);
    }
  }

  int32_t free_row() const {
    for (size_t r = 0; r < rows.size(); ++r)
      if (!rows[r].live) return (int32_t)r;
    return -1;
  }

  void release(Row& row) {
    for (int32_t b : row.blocks) m->free_block(b);
    by_uid.erase(row.uid);
    row = Row{};
  }
};

extern "C" {

rmlx_status rmlx_kv_batch_new(rmlx_block_manager* m, rmlx_prefix_cache* prefix, int32_t max_seqs, rmlx_kv_batch** out) {
  if (!m || !out) return fail(RMLX_E_BAD_ARG, "NULL block manager or out");
  *out = nullptr;
  if (max_seqs <= 0) return fail(RMLX_E_BAD_ARG, "max_seqs must be positive");
  rmlx_kv_batch* b = new (std::nothrow) rmlx_kv_batch{&m->impl, prefix ? &prefix->impl : nullptr, {}, {}, {}};
  if (!b) return fail(RMLX_E_BAD_ARG, "out of host memory");
  b->rows.resize((size_t)max_seqs);
  *out = b;
  return RMLX_OK;
}

void rmlx_kv_batch_destroy(rmlx_kv_batch* b) {
  if (!b) return;
  for (auto& r : b->rows)
    if (r.live) b->release(r);
  delete b;
}

rmlx_status rmlx_kv_batch_add(rmlx_kv_batch* b, uint64_t uid, const uint32_t* prompt, int32_t n, int32_t* row_out,
                              int32_t* cached_tokens, int32_t* slots) {
  if (!b || !prompt || !row_out || !cached_tokens || !slots) return fail(RMLX_E_BAD_ARG, "NULL argument");
  if (n <= 0) return fail(RMLX_E_BAD_ARG, "empty prompt");  // scheduler.rs:214-220
  if (b->by_uid.count(uid)) return fail(RMLX_E_BAD_ARG, "sequence %llu already in the batch", (unsigned long long)uid);
  const int32_t r = b->free_row();
  if (r < 0) return fail(RMLX_E_EXHAUSTED, "batch full (%zu rows)", b->rows.size());
  const int64_t bs = b->bs(), nb = (n + bs - 1) / bs, nfull = n / bs;
  Row row;
  row.uid = uid;
  row.tokens.assign(prompt, prompt + n);
  uint64_t h = 0;
  for (int64_t k = 0; k < nfull; ++k) {
    h = rmlx::xxh::hash_block(h, prompt + k * bs, (int)bs);
    row.hashes.push_back(h);
  }
  int64_t reuse = 0;
  if (b->p) {
    std::vector<int32_t> scratch((size_t)n + 1);
    b->p->lookup(prompt, (size_t)(nfull * bs), scratch.data());
    const int64_t limit = (n - 1) / bs;
    while (reuse < limit) {
      int32_t id;
      if (!b->m->lookup_hash(row.hashes[reuse], &id)) break;
      b->m->increment_ref(id);
      row.blocks.push_back(id);
      reuse += 1;
    }
  }
  for (int64_t k = reuse; k < nb; ++k) {
    int32_t id;
    if (!b->take_block(&id)) {
      for (int32_t x : row.blocks) b->m->free_block(x);
      b->stats.rejected += 1;
      return fail(RMLX_E_EXHAUSTED, "no free block for sequence %llu", (unsigned long long)uid);
    }
    row.blocks.push_back(id);
    const int64_t cnt = std::min<int64_t>(bs, n - k * bs);
    b->m->append_tokens(id, prompt + k * bs, (size_t)cnt);
    if (k < nfull) b->m->register_hash(id, row.hashes[k]);
  }
  b->cache_prefix(prompt, nfull, row.blocks.data());
  const int64_t cached = reuse * bs;
  for (int64_t t = cached; t < n; ++t) slots[t - cached] = (int32_t)(row.blocks[t / bs] * bs + t % bs);
  row.live = true;
  b->rows[r] = std::move(row);
  b->by_uid[uid] = r;
  b->stats.admitted += 1;
  b->stats.prompt_tokens += (uint64_t)n;
  b->stats.cached_tokens += (uint64_t)cached;
  *row_out = r;
  *cached_tokens = (int32_t)cached;
  return RMLX_OK;
}

rmlx_status rmlx_kv_batch_fork(rmlx_kv_batch* b, uint64_t parent, uint64_t child, int32_t* row_out) {
  if (!b || !row_out) return fail(RMLX_E_BAD_ARG, "NULL argument");
  auto it = b->by_uid.find(parent);
  if (it == b->by_uid.end()) return fail(RMLX_E_BAD_ARG, "no sequence %llu", (unsigned long long)parent);
  if (b->by_uid.count(child)) return fail(RMLX_E_BAD_ARG, "sequence %llu already in the batch", (unsigned long long)child);
  const int32_t r = b->free_row();
  if (r < 0) return fail(RMLX_E_EXHAUSTED, "batch full (%zu rows)", b->rows.size());
  Row row = b->rows[it->second];
  row.uid = child;
  for (int32_t x : row.blocks) b->m->increment_ref(x);
  b->rows[r] = std::move(row);
  b->by_uid[child] = r;
  *row_out = r;
  return RMLX_OK;
}

rmlx_status rmlx_kv_batch_remove(rmlx_kv_batch* b, uint64_t uid, int32_t cache_prefix) {
  if (!b) return fail(RMLX_E_BAD_ARG, "NULL batch");
  auto it = b->by_uid.find(uid);
  if (it == b->by_uid.end()) return fail(RMLX_E_BAD_ARG, "no sequence %llu", (unsigned long long)uid);
  Row& row = b->rows[it->second];
  if (cache_prefix) b->cache_prefix(row.tokens.data(), (int64_t)row.hashes.size(), row.blocks.data());
  b->release(row);
  return RMLX_OK;
}

rmlx_status rmlx_kv_batch_step(rmlx_kv_batch* b, const uint64_t* uids, const uint32_t* tokens, int32_t n,
                               int32_t* slots, int32_t* cow_src, int32_t* cow_dst, int32_t* n_cow) {
  if (!b || !n_cow) return fail(RMLX_E_BAD_ARG, "NULL argument");
  *n_cow = 0;
  if (n < 0) return fail(RMLX_E_BAD_ARG, "n < 0");
  if (n == 0) return RMLX_OK;
  if (!uids || !tokens || !slots || !cow_src || !cow_dst) return fail(RMLX_E_BAD_ARG, "NULL argument");
  const int64_t bs = b->bs();
  std::vector<Row*> seq((size_t)n);
  std::unordered_map<uint64_t, int> seen;
  for (int32_t i = 0; i < n; ++i) {
    auto it = b->by_uid.find(uids[i]);
    if (it == b->by_uid.end()) return fail(RMLX_E_BAD_ARG, "no sequence %llu", (unsigned long long)uids[i]);
    if (seen.count(uids[i])) return fail(RMLX_E_BAD_ARG, "sequence %llu listed twice", (unsigned long long)uids[i]);
    seen[uids[i]] = i;
    seq[i] = &b->rows[it->second];
  }
  // what each sequence needs: 0 nothing, 1 a new block, 2 a private copy.
  // A shared tail is copied while other holders remain once the copies
  // planned before it in this step are made: its last holder writes in place.
  std::vector<int> need((size_t)n, 0);
  std::vector<int32_t> got;
  std::unordered_map<int32_t, size_t> copies;
  for (int32_t i = 0; i < n; ++i) {
    const int64_t len = (int64_t)seq[i]->tokens.size();
    if (len % bs == 0) {
      need[i] = 1;
    } else {
      const int32_t tail = seq[i]->blocks.back();
      size_t rc = 0;
      b->m->ref_count(tail, &rc);
      if (rc - copies[tail] > 1) {
        need[i] = 2;
        copies[tail] += 1;
      }
    }
    if (need[i]) {
      int32_t id;
      if (!b->take_block(&id)) {
        for (int32_t x : got) b->m->free_block(x);
        b->stats.new_blocks -= got.size();
        return fail(RMLX_E_EXHAUSTED, "no free block for the step");
      }
      got.push_back(id);
    }
  }
  size_t k = 0;
  for (int32_t i = 0; i < n; ++i) {
    Row& row = *seq[i];
    const int64_t len = (int64_t)row.tokens.size();
    if (need[i] == 1) {
      row.blocks.push_back(got[k++]);
    } else if (need[i] == 2) {
      const int32_t src = row.blocks.back(), dst = got[k++];
      rmlx_block_view v{};
      std::vector<uint32_t> tk((size_t)bs);
      b->m->view(src, &v, tk.data(), tk.size());
      b->m->append_tokens(dst, tk.data(), v.num_filled);
      b->m->free_block(src);  // the copy's source loses this sequence's reference
      row.blocks.back() = dst;
      cow_src[*n_cow] = src;
      cow_dst[*n_cow] = dst;
      *n_cow += 1;
      b->stats.cow_copies += 1;
    }
    const int32_t blk = row.blocks.back();
    slots[i] = (int32_t)(blk * bs + len % bs);
    b->m->append_tokens(blk, tokens + i, 1);
    row.tokens.push_back(tokens[i]);
    if ((len + 1) % bs == 0) {
      const uint64_t parent = row.hashes.empty() ? 0 : row.hashes.back();
      const uint64_t h = rmlx::xxh::hash_block(parent, row.tokens.data() + (len + 1 - bs), (int)bs);
      row.hashes.push_back(h);
      b->m->register_hash(blk, h);
    }
  }
  return RMLX_OK;
}

rmlx_status rmlx_kv_batch_tables(const rmlx_kv_batch* b, int32_t* block_tables, int32_t stride, int32_t* seq_lens,
                                 int32_t max_rows, int32_t* num_rows, int32_t* max_blocks) {
  if (!b || !num_rows || !max_blocks) return fail(RMLX_E_BAD_ARG, "NULL argument");
  int32_t nr = 0, mb = 0;
  for (size_t r = 0; r < b->rows.size(); ++r)
    if (b->rows[r].live) {
      nr = (int32_t)r + 1;
      mb = std::max(mb, (int32_t)b->rows[r].blocks.size());
    }
  *num_rows = nr;
  *max_blocks = mb;
  if (!block_tables && !seq_lens) return RMLX_OK;  // size query
  if (max_rows < nr) return fail(RMLX_E_BAD_ARG, "max_rows %d < %d live rows", max_rows, nr);
  if (block_tables && stride < mb) return fail(RMLX_E_BAD_ARG, "stride %d < %d blocks", stride, mb);
  for (int32_t r = 0; r < nr; ++r) {
    const Row& row = b->rows[r];
    if (seq_lens) seq_lens[r] = row.live ? (int32_t)row.tokens.size() : 0;
    if (block_tables) {
      int32_t* dst = block_tables + (int64_t)r * stride;
      for (int32_t j = 0; j < stride; ++j) dst[j] = (row.live && j < (int32_t)row.blocks.size()) ? row.blocks[j] : 0;
    }
  }
  return RMLX_OK;
}

rmlx_status rmlx_kv_batch_seq(const rmlx_kv_batch* b, uint64_t uid, int32_t* row, int32_t* len, int32_t* block_ids,
                              int32_t cap, int32_t* nblocks) {
  if (!b || !row || !len || !nblocks) return fail(RMLX_E_BAD_ARG, "NULL argument");
  auto it = b->by_uid.find(uid);
  if (it == b->by_uid.end()) return fail(RMLX_E_BAD_ARG, "no sequence %llu", (unsigned long long)uid);
  const Row& r = b->rows[it->second];
  *row = it->second;
  *len = (int32_t)r.tokens.size();
  *nblocks = (int32_t)r.blocks.size();
  if (block_ids)
    for (int32_t j = 0; j < cap && j < (int32_t)r.blocks.size(); ++j) block_ids[j] = r.blocks[j];
  return RMLX_OK;
}

void rmlx_kv_batch_stats(const rmlx_kv_batch* b, rmlx_batch_stats* out) {
  if (b && out) *out = b->stats;
}

int32_t rmlx_kv_batch_num_active(const rmlx_kv_batch* b) {
  return b ? (int32_t)b->by_uid.size() : 0;
}

rmlx_status rmlx_kv_batch_rows(const rmlx_kv_batch* b, uint64_t* uids, int32_t* live, int32_t cap, int32_t* num_rows) {
  if (!b || !num_rows) return fail(RMLX_E_BAD_ARG, "NULL batch or num_rows");
  *num_rows = (int32_t)b->rows.size();
  for (int32_t r = 0; r < cap && r < *num_rows; ++r) {
    if (uids) uids[r] = b->rows[r].live ? b->rows[r].uid : 0;
    if (live) live[r] = b->rows[r].live ? 1 : 0;
  }
  return RMLX_OK;
}

}  // extern "C"
