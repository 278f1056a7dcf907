// Host-side paged block manager (the drop-in for PagedCacheManager,
// crates/rmlx-serve-cache/src/paged_cache.rs:71-302); see block_manager.cc.
#pragma once

#include "common.h"

namespace rmlx {

class BlockManager {
 public:
  BlockManager(size_t block_size, size_t num_blocks)
      : bs_(block_size),
        n_(num_blocks),
        ring_(num_blocks),
        ref_(num_blocks, 0),
        filled_(num_blocks, 0),
        has_hash_(num_blocks, 0),
        hash_(num_blocks, 0),
        tokens_(num_blocks * block_size) {
    for (size_t i = 0; i < n_; ++i) ring_[i] = (int32_t)i;  // paged_cache.rs:95
    head_ = 0;
    count_ = n_;
  }

  bool valid(int32_t id) const { return id >= 0 && (size_t)id < n_; }

  bool allocate(int32_t* out) {  // paged_cache.rs:110-115
    if (count_ == 0) return false;
    int32_t id = ring_[head_];
    head_ = head_ + 1 == n_ ? 0 : head_ + 1;
    --count_;
    reset(id);
    ref_[id] = 1;
    *out = id;
    return true;
  }

  rmlx_status free_block(int32_t id) {  // paged_cache.rs:125-149
    if (!valid(id)) return fail(RMLX_E_RANGE, "block_id %d out of range (num_blocks = %zu)", id, n_);
    if (ref_[id] == 0) return fail(RMLX_E_DOUBLE_FREE, "double free: block %d already has ref_count 0", id);
    if (--ref_[id] == 0) {
      if (has_hash_[id]) {
        int32_t holder;
        if (index_.find(hash_[id], &holder) && holder == id) index_.erase(hash_[id]);
      }
      reset(id);
      size_t tail = head_ + count_;
      if (tail >= n_) tail -= n_;
      ring_[tail] = id;
      ++count_;
    }
    return RMLX_OK;
  }

  rmlx_status ref_count(int32_t id, size_t* out) const {  // :157-163
    if (!valid(id)) return fail(RMLX_E_RANGE, "block_id %d out of range", id);
    *out = ref_[id];
    return RMLX_OK;
  }

  rmlx_status increment_ref(int32_t id) {  // :172-182
    if (!valid(id)) return fail(RMLX_E_RANGE, "block_id %d out of range", id);
    if (ref_[id] == 0) return fail(RMLX_E_FREE_BLOCK, "cannot increment ref on free block %d", id);
    ++ref_[id];
    return RMLX_OK;
  }

  rmlx_status copy_on_write(int32_t id, int32_t* nid, int32_t* copied) {  // :197-224
    *copied = 0;
    if (!valid(id)) return fail(RMLX_E_RANGE, "block_id %d out of range", id);
    if (ref_[id] <= 1) return RMLX_OK;
    int32_t n;
    if (!allocate(&n)) return RMLX_OK;
    memcpy(&tokens_[(size_t)n * bs_], &tokens_[(size_t)id * bs_], filled_[id] * sizeof(uint32_t));
    filled_[n] = filled_[id];
    has_hash_[n] = 0;
    --ref_[id];
    *nid = n;
    *copied = 1;
    return RMLX_OK;
  }

  rmlx_status register_hash(int32_t id, uint64_t h) {  // :265-272
    if (!valid(id)) return fail(RMLX_E_RANGE, "block_id %d out of range", id);
    has_hash_[id] = 1;
    hash_[id] = h;
    index_.put(h, id);
    return RMLX_OK;
  }

  bool lookup_hash(uint64_t h, int32_t* out) const {  // :278-282
    int32_t id;
    if (!index_.find(h, &id) || ref_[id] == 0) return false;
    *out = id;
    return true;
  }

  rmlx_status append_tokens(int32_t id, const uint32_t* t, size_t k) {  // :288-301
    if (!valid(id)) return fail(RMLX_E_RANGE, "block_id %d out of range", id);
    if (filled_[id] + k > bs_)
      return fail(RMLX_E_OVERFLOW, "block %d overflow: %u filled + %zu new > %zu block_size", id, filled_[id], k,
                  bs_);
    if (k) memcpy(&tokens_[(size_t)id * bs_ + filled_[id]], t, k * sizeof(uint32_t));
    filled_[id] += (uint32_t)k;
    has_hash_[id] = 0;
    return RMLX_OK;
  }

  bool view(int32_t id, rmlx_block_view* v, uint32_t* tok, size_t cap) const {  // :249-251
    if (!valid(id)) return false;
    v->block_id = id;
    v->ref_count = ref_[id];
    v->has_hash = has_hash_[id];
    v->hash = hash_[id];
    v->num_filled = filled_[id];
    for (size_t i = 0; i < filled_[id] && i < cap; ++i) tok[i] = tokens_[(size_t)id * bs_ + i];
    return true;
  }

  size_t num_free() const { return count_; }
  size_t num_blocks() const { return n_; }
  size_t block_size() const { return bs_; }

 private:
  void reset(int32_t id) {  // KVCacheBlock::reset, paged_cache.rs:51-56
    ref_[id] = 0;
    has_hash_[id] = 0;
    hash_[id] = 0;
    filled_[id] = 0;
  }
  size_t bs_, n_;
  std::vector<int32_t> ring_;
  size_t head_ = 0, count_ = 0;
  std::vector<uint32_t> ref_, filled_;
  std::vector<uint8_t> has_hash_;
  std::vector<uint64_t> hash_;
  std::vector<uint32_t> tokens_;
  FlatMap64 index_;
};

}  // namespace rmlx

struct rmlx_block_manager {
  rmlx::BlockManager impl;
  rmlx_block_manager(size_t bs, size_t n) : impl(bs, n) {}
};
