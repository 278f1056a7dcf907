// Prefix-block chain hash, shared by the GPU kernel (kv_hash.cu) and the
// host batch planner (kv_batch.cc):
//   hash[b] = XXH64(le64(hash[b-1]) || le32(token ids of block b), seed 0)
// XXH64 is Y. Collet's published 64-bit hash, restated from its
// specification for word-aligned messages (the message is 8 + 4 * count
// bytes).
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define RMLX_HD __host__ __device__ __forceinline__
#else
#define RMLX_HD inline
#endif

namespace rmlx {
namespace xxh {
constexpr uint64_t P1 = 0x9E3779B185EBCA87ULL, P2 = 0xC2B2AE3D27D4EB4FULL, P3 = 0x165667B19E3779F9ULL,
                   P4 = 0x85EBCA77C2B2AE63ULL, P5 = 0x27D4EB2F165667C5ULL;
RMLX_HD uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
RMLX_HD uint64_t round1(uint64_t acc, uint64_t lane) { return rotl(acc + lane * P2, 31) * P1; }
RMLX_HD uint64_t merge(uint64_t acc, uint64_t v) { return (acc ^ round1(0, v)) * P1 + P4; }

RMLX_HD uint32_t load(const uint32_t* p) {
#if defined(__CUDA_ARCH__)
  return __ldg(p);
#else
  return *p;
#endif
}

// Message word i: 0,1 = the parent hash (little-endian halves), 2.. = tokens.
struct Msg {
  uint64_t parent;
  const uint32_t* tok;
  RMLX_HD uint32_t word(int i) const {
    return i == 0 ? (uint32_t)parent : (i == 1 ? (uint32_t)(parent >> 32) : load(tok + (i - 2)));
  }
  RMLX_HD uint64_t lane(int i) const { return (uint64_t)word(i) | ((uint64_t)word(i + 1) << 32); }
};

RMLX_HD uint64_t hash_block(uint64_t parent, const uint32_t* tok, int count) {
  const Msg m{parent, tok};
  const int nw = 2 + count;
  const uint64_t len = 4ull * (uint64_t)nw;
  int p = 0;
  uint64_t h;
  if (len >= 32) {
    uint64_t v1 = P1 + P2, v2 = P2, v3 = 0, v4 = 0 - P1;
    while (nw - p >= 8) {
      v1 = round1(v1, m.lane(p));
      v2 = round1(v2, m.lane(p + 2));
      v3 = round1(v3, m.lane(p + 4));
      v4 = round1(v4, m.lane(p + 6));
      p += 8;
    }
    h = rotl(v1, 1) + rotl(v2, 7) + rotl(v3, 12) + rotl(v4, 18);
    h = merge(h, v1);
    h = merge(h, v2);
    h = merge(h, v3);
    h = merge(h, v4);
  } else {
    h = P5;
  }
  h += len;
  while (nw - p >= 2) {
    h ^= round1(0, m.lane(p));
    h = rotl(h, 27) * P1 + P4;
    p += 2;
  }
  if (nw - p >= 1) {
    h ^= (uint64_t)m.word(p) * P1;
    h = rotl(h, 23) * P2 + P3;
  }
  h ^= h >> 33;
  h *= P2;
  h ^= h >> 29;
  h *= P3;
  h ^= h >> 32;
  return h;
}
}  // namespace xxh
}  // namespace rmlx
