// Host-side prefix cache (the drop-in for PrefixCacheManager,
// crates/rmlx-serve-cache/src/prefix_cache.rs:44-292, and
// MemoryAwarePrefixCache, memory.rs:10-200); see prefix_cache.cc.
#pragma once

#include <deque>
#include <set>
#include <tuple>

#include "common.h"

namespace rmlx {

class PrefixTrie {
 public:
  explicit PrefixTrie(size_t max_blocks) : max_blocks_(max_blocks) { new_node(UINT32_MAX, 0); }

  // lookup -- prefix_cache.rs:85-113
  size_t lookup(const uint32_t* tokens, size_t n, int32_t* out) {
    total_lookups_ += 1;
    lookup_tokens_ += n;
    uint64_t t = ++clock_;
    uint32_t cur = 0;
    size_t k = 0;
    for (size_t i = 0; i < n; ++i) {
      int32_t child;
      if (!children_.find(edge(cur, tokens[i]), &child)) break;
      cur = (uint32_t)child;
      touch(cur, t);
      if (has_block_[cur]) out[k++] = block_[cur];
    }
    hit_tokens_ += k;
    return k;
  }

  // insert -- prefix_cache.rs:126-179
  void insert(const uint32_t* tokens, size_t n, const int32_t* ids, size_t nb) {
    insert_report(tokens, n, ids, nb, nullptr, nullptr);
  }

  // insert, also reporting per block index whether its boundary node had no
  // block before (attached[i] = 1) and which block it replaced (replaced[i],
  // -1 for none).  The admission driver uses this to keep the cache's own
  // reference counts on the blocks it holds.
  void insert_report(const uint32_t* tokens, size_t n, const int32_t* ids, size_t nb, uint8_t* attached,
                     int32_t* replaced) {
    if (attached)
      for (size_t i = 0; i < nb; ++i) attached[i] = 0;
    if (replaced)
      for (size_t i = 0; i < nb; ++i) replaced[i] = -1;
    if (n == 0 || nb == 0) return;
    size_t tpb = nb == 1 ? n : n / nb;
    uint64_t t = ++clock_;
    uint32_t cur = 0;
    size_t bi = 0;
    for (size_t i = 0; i < n; ++i) {
      int32_t child;
      uint32_t next;
      if (children_.find(edge(cur, tokens[i]), &child)) {
        next = (uint32_t)child;
      } else {
        next = new_node(cur, tokens[i]);
        children_.put(edge(cur, tokens[i]), (int32_t)next);
        if (nchild_[cur]++ == 0) reclassify(cur);  // cur stops being a leaf
      }
      touch(next, t);
      bool boundary = false;
      if (bi < nb) boundary = (bi == nb - 1) ? (i == n - 1) : ((i + 1) == (bi + 1) * tpb);
      if (boundary) {
        if (has_block_[next]) {
          if (replaced && block_[next] != ids[bi]) replaced[bi] = block_[next];
          block_[next] = ids[bi];
        } else {
          has_block_[next] = 1;
          block_[next] = ids[bi];
          order_.insert(key(next));
          num_blocks_ += 1;
          if (attached) attached[bi] = 1;
        }
        bi += 1;
      }
      cur = next;
    }
  }

  // evict_lru -- prefix_cache.rs:187-232
  bool evict_lru(int32_t* out) {
    if (num_blocks_ == 0 || order_.empty()) return false;
    auto it = order_.begin();
    uint32_t idx = std::get<2>(*it);
    bool leaf = std::get<0>(*it) == 0;
    order_.erase(it);
    *out = block_[idx];
    has_block_[idx] = 0;
    num_blocks_ -= 1;
    if (leaf) prune_leaf(idx);
    return true;
  }

  double hit_rate() const {  // :266-271
    return lookup_tokens_ == 0 ? 0.0 : (double)hit_tokens_ / (double)lookup_tokens_;
  }
  size_t num_blocks() const { return num_blocks_; }
  size_t max_blocks() const { return max_blocks_; }
  bool is_full() const { return num_blocks_ >= max_blocks_; }
  size_t num_nodes() const { return parent_.size(); }

 private:
  using Key = std::tuple<uint8_t, uint64_t, uint32_t>;  // (is_internal, last_access, index)
  static uint64_t edge(uint32_t parent, uint32_t token) { return ((uint64_t)parent << 32) | token; }
  Key key(uint32_t i) const { return Key(nchild_[i] ? 1 : 0, last_[i], i); }

  uint32_t new_node(uint32_t parent, uint32_t token) {
    uint32_t i = (uint32_t)parent_.size();
    parent_.push_back(parent);
    token_.push_back(token);
    nchild_.push_back(0);
    has_block_.push_back(0);
    block_.push_back(0);
    last_.push_back(0);
    return i;
  }
  void touch(uint32_t i, uint64_t t) {
    if (last_[i] == t) return;
    if (has_block_[i]) {
      order_.erase(key(i));
      last_[i] = t;
      order_.insert(key(i));
    } else {
      last_[i] = t;
    }
  }
  // Called after nchild_[i] crossed 0 <-> 1: move i to its new class.
  void reclassify(uint32_t i) {
    if (!has_block_[i]) return;
    Key old(nchild_[i] ? 0 : 1, last_[i], i);
    order_.erase(old);
    order_.insert(key(i));
  }
  void prune_leaf(uint32_t i) {  // :235-260
    if (i == 0 || nchild_[i] != 0 || has_block_[i]) return;
    uint32_t p = parent_[i];
    children_.erase(edge(p, token_[i]));
    if (--nchild_[p] == 0) reclassify(p);
  }

  size_t max_blocks_;
  size_t num_blocks_ = 0;
  uint64_t clock_ = 0, total_lookups_ = 0, hit_tokens_ = 0, lookup_tokens_ = 0;
  std::vector<uint32_t> parent_, token_, nchild_;
  std::vector<uint8_t> has_block_;
  std::vector<int32_t> block_;
  std::vector<uint64_t> last_;
  FlatMap64 children_;
  std::set<Key> order_;
};

// memory.rs:10-200 with available_memory_mb() == usize::MAX (:88-91).
class MemoryAwarePrefix {
 public:
  MemoryAwarePrefix(size_t max_blocks, size_t limit_mb, size_t bpb)
      : trie_(max_blocks), limit_(limit_mb * 1024 * 1024), bpb_(bpb) {}
  bool should_evict() const {  // :99-110
    if (usage_ >= limit_) return true;
    if (trie_.is_full()) return true;
    size_t available_mb = SIZE_MAX;
    size_t thr = limit_ / (1024 * 1024) / 10;
    return available_mb < (thr > 256 ? thr : 256);
  }
  void evict_until_threshold() {  // :117-136
    size_t target = (size_t)((double)limit_ * 0.8);
    while (usage_ > target) {
      int32_t id;
      if (!trie_.evict_lru(&id)) break;
      usage_ = usage_ > bpb_ ? usage_ - bpb_ : 0;
      evicted_.push_back(id);
    }
  }
  void insert(const uint32_t* t, size_t n, const int32_t* ids, size_t nb) {  // :149-158
    if (should_evict()) evict_until_threshold();
    trie_.insert(t, n, ids, nb);
    usage_ += nb * bpb_;
  }
  bool evict_lru(int32_t* out) {  // :161-168
    bool ok = trie_.evict_lru(out);
    if (ok) usage_ = usage_ > bpb_ ? usage_ - bpb_ : 0;
    return ok;
  }
  size_t drain(int32_t* out, size_t cap) {
    size_t k = 0;
    while (k < cap && !evicted_.empty()) {
      out[k++] = evicted_.front();
      evicted_.pop_front();
    }
    return k;
  }
  PrefixTrie trie_;
  size_t limit_, usage_ = 0, bpb_;
  std::deque<int32_t> evicted_;
};

}  // namespace rmlx

struct rmlx_prefix_cache {
  rmlx::PrefixTrie impl;
  explicit rmlx_prefix_cache(size_t m) : impl(m) {}
};
struct rmlx_mem_prefix_cache {
  rmlx::MemoryAwarePrefix impl;
  rmlx_mem_prefix_cache(size_t m, size_t mb, size_t bpb) : impl(m, mb, bpb) {}
};
