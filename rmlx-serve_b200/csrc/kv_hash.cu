// Prefix-block chain hash on the GPU.
//
// The reference's PagedCacheManager indexes blocks by caller-supplied 64-bit
// content hashes (crates/rmlx-serve-cache/src/paged_cache.rs:265-282) and no
// code in the reference computes one.  This file defines them:
//   hash[b] = XXH64(le64(hash[b-1]) || le32(token ids of block b), seed 0)
// with hash[-1] = the request's root hash (XXH64 in chain_hash.h).
//
// One thread walks one request's chain (block b depends on block b-1); the
// token reads of a block are 64 contiguous bytes.
#include "chain_hash.h"
#include "device_common.cuh"

namespace rmlx {

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
