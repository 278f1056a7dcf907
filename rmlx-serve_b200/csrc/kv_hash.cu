// Prefix-block chain hash on the GPU.
//
// The reference's PagedCacheManager indexes blocks by caller-supplied 64-bit
// content hashes (crates/rmlx-serve-cache/src/paged_cache.rs:265-282) and no
// code in the reference computes one.  This file defines them:
//   hash[b] = XXH64(le64(hash[b-1]) || le32(token ids of block b), seed 0)
// with hash[-1] = the request's root hash.  XXH64 is Y. Collet's published
// 64-bit hash; it is restated here from its specification for word-aligned
// messages (the message is 8 + 4 * count bytes).
//
// One thread walks one request's chain (block b depends on block b-1); the
// token reads of a block are 64 contiguous bytes.
#include "device_common.cuh"

namespace rmlx {
namespace xxh {
constexpr uint64_t P1 = 0x9E3779B185EBCA87ULL, P2 = 0xC2B2AE3D27D4EB4FULL, P3 = 0x165667B19E3779F9ULL,
                   P4 = 0x85EBCA77C2B2AE63ULL, P5 = 0x27D4EB2F165667C5ULL;
__device__ __forceinline__ uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
__device__ __forceinline__ uint64_t round1(uint64_t acc, uint64_t lane) { return rotl(acc + lane * P2, 31) * P1; }
__device__ __forceinline__ uint64_t merge(uint64_t acc, uint64_t v) { return (acc ^ round1(0, v)) * P1 + P4; }

// Message word i: 0,1 = the parent hash (little-endian halves), 2.. = tokens.
struct Msg {
  uint64_t parent;
  const uint32_t* tok;
  __device__ __forceinline__ uint32_t word(int i) const {
    return i == 0 ? (uint32_t)parent : (i == 1 ? (uint32_t)(parent >> 32) : __ldg(tok + (i - 2)));
  }
  __device__ __forceinline__ uint64_t lane(int i) const { return (uint64_t)word(i) | ((uint64_t)word(i + 1) << 32); }
};

__device__ uint64_t hash_block(uint64_t parent, const uint32_t* tok, int count) {
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

__global__ void __launch_bounds__(128) hash_chains_kernel(const uint32_t* __restrict__ tokens,
                                                          const int64_t* __restrict__ cu_tokens,
                                                          const uint64_t* __restrict__ root, int nreq, int bs,
                                                          const int64_t* __restrict__ cu_blocks,
                                                          uint64_t* __restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= nreq) return;
  const int64_t t0 = cu_tokens[r], n = cu_tokens[r + 1] - t0;
  if (n <= 0) return;
  // Never write past this request's slice of `out`, whatever cu_blocks says.
  const int64_t nb = min((n + bs - 1) / bs, cu_blocks[r + 1] - cu_blocks[r]);
  uint64_t parent = root ? root[r] : 0ull;
  uint64_t* o = out + cu_blocks[r];
  for (int64_t b = 0; b < nb; ++b) {
    const int cnt = (int)min((int64_t)bs, n - b * bs);
    parent = xxh::hash_block(parent, tokens + t0 + b * bs, cnt);
    o[b] = parent;
  }
}

}  // namespace rmlx

using namespace rmlx;

extern "C" rmlx_status rmlx_hash_block_chains(const uint32_t* tokens, const int64_t* cu_tokens,
                                              const uint64_t* root_hashes, int32_t num_requests, int32_t block_size,
                                              const int64_t* cu_blocks, uint64_t* out, void* stream) {
  if (num_requests < 0 || block_size <= 0) return fail(RMLX_E_BAD_ARG, "num_requests < 0 or block_size <= 0");
  if (num_requests == 0) return RMLX_OK;
  if (!tokens || !cu_tokens || !cu_blocks || !out) return fail(RMLX_E_BAD_ARG, "NULL device array");
  const int grid = (num_requests + 127) / 128;
  hash_chains_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(tokens, cu_tokens, root_hashes, num_requests, block_size,
                                                             cu_blocks, out);
  return cuda_check(cudaGetLastError(), "hash_chains launch");
}
