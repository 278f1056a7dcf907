// Shared helpers for the rmlx_kv library: status plumbing and a small
// open-addressing hash map used by the host-side indices.
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "rmlx_kv.h"

namespace rmlx {

// Records a thread-local message for rmlx_last_error() and returns `s`.
rmlx_status fail(rmlx_status s, const char* fmt, ...);
void clear_error();

// Linear-probing map from a 64-bit key to a 32-bit value with backward-shift
// deletion (no tombstones).  Keys are mixed with a 64-bit finaliser before
// probing so that sequential keys spread.  Grows at 50% load.
class FlatMap64 {
 public:
  FlatMap64() { rehash(16); }
  bool find(uint64_t key, int32_t* val) const {
    size_t i = slot(key);
    while (used_[i]) {
      if (keys_[i] == key) {
        *val = vals_[i];
        return true;
      }
      i = (i + 1) & mask_;
    }
    return false;
  }
  // Inserts or overwrites.
  void put(uint64_t key, int32_t val) {
    if ((size_ + 1) * 2 > cap_) rehash(cap_ * 2);
    size_t i = slot(key);
    while (used_[i]) {
      if (keys_[i] == key) {
        vals_[i] = val;
        return;
      }
      i = (i + 1) & mask_;
    }
    used_[i] = 1;
    keys_[i] = key;
    vals_[i] = val;
    ++size_;
  }
  bool erase(uint64_t key) {
    size_t i = slot(key);
    while (used_[i]) {
      if (keys_[i] == key) {
        erase_at(i);
        return true;
      }
      i = (i + 1) & mask_;
    }
    return false;
  }
  size_t size() const { return size_; }
  void reserve(size_t n) {
    size_t c = cap_;
    while (n * 2 > c) c *= 2;
    if (c != cap_) rehash(c);
  }

 private:
  static uint64_t mix(uint64_t x) {
    x ^= x >> 31;
    x *= 0x7fb5d329728ea185ULL;
    x ^= x >> 27;
    x *= 0x81dadef4bc2dd44dULL;
    x ^= x >> 33;
    return x;
  }
  size_t slot(uint64_t key) const { return (size_t)mix(key) & mask_; }
  void erase_at(size_t i) {
    // Backward-shift: pull later entries of the same probe run into the hole.
    size_t hole = i;
    size_t j = i;
    for (;;) {
      j = (j + 1) & mask_;
      if (!used_[j]) break;
      size_t home = slot(keys_[j]);
      // Move j into the hole if its home is not in (hole, j] cyclically.
      bool between = (hole <= j) ? (home > hole && home <= j) : (home > hole || home <= j);
      if (!between) {
        keys_[hole] = keys_[j];
        vals_[hole] = vals_[j];
        hole = j;
      }
    }
    used_[hole] = 0;
    --size_;
  }
  void rehash(size_t cap) {
    std::vector<uint64_t> ok;
    std::vector<int32_t> ov;
    std::vector<uint8_t> ou;
    ok.swap(keys_);
    ov.swap(vals_);
    ou.swap(used_);
    cap_ = cap;
    mask_ = cap - 1;
    keys_.assign(cap, 0);
    vals_.assign(cap, 0);
    used_.assign(cap, 0);
    size_ = 0;
    for (size_t i = 0; i < ou.size(); ++i)
      if (ou[i]) put(ok[i], ov[i]);
  }
  std::vector<uint64_t> keys_;
  std::vector<int32_t> vals_;
  std::vector<uint8_t> used_;
  size_t cap_ = 0, mask_ = 0, size_ = 0;
};

}  // namespace rmlx
