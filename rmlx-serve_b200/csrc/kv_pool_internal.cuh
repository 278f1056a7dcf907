// Internals shared by the pool's CUDA sources (not part of the C ABI): the
// pool object, its device-side geometry, the per-CTA sequence-length scan
// and launch helpers.
#pragma once
#include "device_common.cuh"

namespace rmlx {

struct PoolGeo {
  uint8_t* base;
  int64_t tile_bytes;
  int32_t layers, heads, bs, nblocks;
  int32_t row_bytes, meta_row_bytes;
  int32_t dtype;  // RMLX_BF16 / RMLX_F16 / RMLX_F32 of the stored (or dequantised) rows
  __device__ __forceinline__ int64_t tile_off(int64_t blk, int l, int kv, int h) const {
    return (((blk * layers + l) * 2 + kv) * heads + h) * tile_bytes;
  }
};

// ---------------------------------------------------------------------------
// Per-CTA prologue of the gathers: exclusive prefix sums of blocks per
// sequence (cub) and of tokens (cut) over seq_lens, into shared memory.
// ---------------------------------------------------------------------------
static __device__ void scan_seq_lens(const int32_t* __restrict__ lens, int n, int bs, int32_t* cub, int32_t* cut) {
  __shared__ int32_t wsb[32], wst[32];
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, w = tid >> 5, nw = nt >> 5;
  const int per = (n + nt - 1) / nt;
  const int beg = min(n, tid * per), end = min(n, beg + per);
  int32_t sb = 0, st = 0;
  for (int i = beg; i < end; ++i) {
    int32_t L = max(__ldg(lens + i), 0);
    sb += (L + bs - 1) / bs;
    st += L;
  }
  int32_t xb = sb, xt = st;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int32_t yb = __shfl_up_sync(0xffffffffu, xb, o), yt = __shfl_up_sync(0xffffffffu, xt, o);
    if (lane >= o) {
      xb += yb;
      xt += yt;
    }
  }
  if (lane == 31) {
    wsb[w] = xb;
    wst[w] = xt;
  }
  __syncthreads();
  if (w == 0) {
    int32_t vb = lane < nw ? wsb[lane] : 0, vt = lane < nw ? wst[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int32_t yb = __shfl_up_sync(0xffffffffu, vb, o), yt = __shfl_up_sync(0xffffffffu, vt, o);
      if (lane >= o) {
        vb += yb;
        vt += yt;
      }
    }
    wsb[lane] = vb;
    wst[lane] = vt;
  }
  __syncthreads();
  int32_t pb = xb - sb + (w ? wsb[w - 1] : 0), pt = xt - st + (w ? wst[w - 1] : 0);
  for (int i = beg; i < end; ++i) {
    cub[i] = pb;
    cut[i] = pt;
    int32_t L = max(__ldg(lens + i), 0);
    pb += (L + bs - 1) / bs;
    pt += L;
  }
  if (tid == 0) {
    cub[n] = wsb[nw - 1];
    cut[n] = wst[nw - 1];
  }
  __syncthreads();
}

// Largest s in [0, n) with cub[s] <= gi (cub is non-decreasing, cub[0] = 0).
__device__ __forceinline__ int find_seq(const int32_t* cub, int n, int64_t gi) {
  int lo = 0, hi = n;  // invariant: cub[lo] <= gi < cub[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (cub[mid] <= gi) lo = mid;
    else hi = mid;
  }
  return lo;
}

}  // namespace rmlx

struct rmlx_kv_pool {
  rmlx_pool_config cfg;
  int device = 0;
  uint8_t* base = nullptr;
  int32_t* err = nullptr;
  size_t bytes = 0, tile_bytes = 0, block_bytes = 0, row_bytes = 0, meta_row_bytes = 0;
  int num_sms = 148;
  // Persistent-grid size of this pool's gather kernel for the last dynamic
  // shared-memory size used (the kernel is fixed by the pool's config).
  size_t gather_smem = 0;
  int gather_grid = 0;
  // Work-item counter of the decode attention (zero between launches).
  unsigned long long* attn_work = nullptr;
  // The decode attention's launch shape for the last (num_seqs, q_heads_per_kv):
  // split kernel, its dynamic shared memory, grid and work-item target.
  int attn_nseq = -1, attn_G = -1, attn_grid = 0;
  void* attn_fn = nullptr;
  size_t attn_smem = 0;
  int64_t attn_target = 0;
  rmlx::PoolGeo geo() const {
    rmlx::PoolGeo g;
    g.base = base;
    g.tile_bytes = (int64_t)tile_bytes;
    g.layers = cfg.num_layers;
    g.heads = cfg.num_kv_heads;
    g.bs = cfg.block_size;
    g.nblocks = cfg.num_blocks;
    g.row_bytes = (int32_t)row_bytes;
    g.meta_row_bytes = (int32_t)meta_row_bytes;
    g.dtype = cfg.dtype;
    return g;
  }
};

namespace rmlx {

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }
inline bool is_pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }
inline int log2i(int x) {
  int r = 0;
  while ((1 << r) < x) ++r;
  return r;
}

// Persistent grid: resident CTAs per SM x SM count.
template <typename K>
int persistent_grid(K kernel, int threads, size_t smem, int num_sms) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  return per_sm * num_sms;
}

template <typename K>
rmlx_status prepare_smem(K kernel, size_t smem) {
  if (smem <= 48 * 1024) return RMLX_OK;
  return cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "cudaFuncSetAttribute");
}

}  // namespace rmlx
