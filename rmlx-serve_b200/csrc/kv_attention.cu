// Paged decode attention over the pool: the consumer of the K/V tiles, reading
// them in place instead of through a gathered copy.
//
// For each sequence s and query head j (grouped: q heads g*G .. g*G+G-1 share
// KV head g of this pool), out = softmax(scale * q K^T) V over the sequence's
// len tokens, K/V rows located through the block table exactly like the
// gather (token t: block bt[s][t / block_size], row t % block_size).
//
// Split over the sequence (flash-decoding): a work item is (split of 256
// down to 64 tokens, KV head), one warp per item, items handed out by a
// counter.  A warp streams its split in chunks of 16 tokens through shared
// memory (cp.async) and runs both products on the tensor cores with
// mma.sync m16n8k16 (f16/bf16 inputs, f32 accumulation), with an online
// softmax in the log2 domain.  A sequence held by one item is normalised
// and written directly; otherwise each item writes its unnormalised O, max
// and sum to a workspace, and a second kernel combines the splits of each
// (sequence, query head) and writes the output in the pool's type.
//
// Three split kernels:
//   * paged_decode_attn_rows_kernel (bf16/f16 pools): tokens are the M rows
//     and the query heads the N columns of both products (S^T = K Q^T,
//     O^T += V^T P^T), the queries held in registers;
//   * paged_decode_attn_codes_kernel (quantised pools whose groups span
//     whole k-steps): the same orientation, fed the 4/8-bit codes as exact
//     f16 integers, with scale and zero applied around the products;
//   * paged_decode_attn_kernel (quantised pools with smaller groups): the
//     query heads as the M rows, K and V dequantised into a shared-memory
//     tile first.
//
// The work is HBM-bound by arithmetic intensity: per token and KV head a
// bf16 pool reads 2 x head_dim x 2 bytes for 4 x G x head_dim flops (G =
// 4..8: 8..16 flops per byte), two orders of magnitude under the tensor
// cores' ridge point, so the warp-level mma is not the limit; what matters
// is that every K/V byte is read once with enough bytes in flight, and, for
// quantised pools, how few instructions each code costs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "dequant.cuh"
#include "kv_pool_internal.cuh"

namespace rmlx {

constexpr int ATT_SPLIT = 256;  // tokens per work item
constexpr int ATT_CHUNK = 16;   // tokens per tensor-core step
constexpr int ATT_WARPS = 4;    // warps per CTA (independent items)

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int DT>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if (DT == RMLX_BF16) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
// 16-byte async copy; src_bytes = 0 fills the destination with zeros and reads nothing.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// 4- and 8-byte async copies (short scale/zero rows), same zero-fill rule.
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int DT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if (DT == RMLX_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Combine the splits of sequence s for query head j of KV head h: n splits
// starting at global split `base` (items (base + i) * heads + h), written as
// out[s][h * G + j][:] in the pool's type.  Splits are taken 16 at a time:
// their (max, sum) pairs one per lane, and every lane's head_dim / 32
// elements of the 16 partial outputs, all loaded before any arithmetic, so a
// round costs one memory latency; weights reach the lanes by shuffle and an
// online max carries across rounds.
template <int HD>
__device__ __forceinline__ void merge_splits(const float* part_o, const float* part_ml, int h, int j, int G,
                                             int heads, int base, int k0, int kstep, int nk, int lane, float& mx,
                                             float& L, float* acc) {
  // splits base + k0 + t * kstep, t < nk, into the running (mx, L, acc);
  // L is held as per-lane shares (each lane's own splits), acc as this
  // lane's head_dim / 32 elements
  constexpr int EPL = HD / 32;
  constexpr int R = 16;
  constexpr unsigned FULL = 0xffffffffu;
  const float2* ml = reinterpret_cast<const float2*>(part_ml) + ((int64_t)base * heads + h) * G + j;
  const int64_t mstride = (int64_t)heads * G;
  const float* po = part_o + (((int64_t)base * heads + h) * G + j) * HD + lane * EPL;
  const int64_t ostride = (int64_t)heads * G * HD;
  for (int r0 = 0; r0 < nk; r0 += R) {
    const int cnt = min(R, nk - r0);
    float2 mlv = make_float2(-INFINITY, 0.0f);
    if (lane < cnt) mlv = __ldcg(ml + (int64_t)(k0 + (r0 + lane) * kstep) * mstride);
    float vv[R][EPL];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const float* pk = po + (int64_t)(k0 + (r0 + k) * kstep) * ostride;
#pragma unroll
      for (int e = 0; e < EPL; e += 2) {
        float2 x = make_float2(0.0f, 0.0f);
        if (k < cnt) x = __ldcg(reinterpret_cast<const float2*>(pk + e));
        vv[k][e] = x.x;
        vv[k][e + 1] = x.y;
      }
    }
    float cm = mlv.x;
#pragma unroll
    for (int o = 16; o; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(FULL, cm, o));
    const float nm = fmaxf(mx, cm);
    const float a = ex2(mx - nm);
    L *= a;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] *= a;
    mx = nm;
    const float wl = lane < cnt ? ex2(mlv.x - nm) : 0.0f;
    L += mlv.y * wl;
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const float w = __shfl_sync(FULL, wl, k);
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[e] += w * vv[k][e];
    }
  }
}

template <int DT, int HD>
__device__ __forceinline__ void store_out_row(uint8_t* out, int s, int h, int j, int G, int heads, const float* acc,
                                              float inv, int lane) {
  constexpr int EPL = HD / 32;
  uint32_t wv[EPL / 2];
#pragma unroll
  for (int e = 0; e < EPL; e += 2) wv[e / 2] = pack2<DT>(acc[e] * inv, acc[e + 1] * inv);
  uint8_t* dst = out + ((int64_t)s * heads * G + (int64_t)h * G + j) * HD * 2 + lane * EPL * 2;
  if (EPL == 4) *reinterpret_cast<uint2*>(dst) = make_uint2(wv[0], wv[1]);
  else *reinterpret_cast<uint32_t*>(dst) = wv[0];
}

template <int DT, int HD>
__device__ __forceinline__ void combine_splits(const float* part_o, const float* part_ml, uint8_t* out, int s,
                                               int h, int j, int G, int heads, int base, int n, int lane) {
  constexpr int EPL = HD / 32;
  constexpr unsigned FULL = 0xffffffffu;
  float mx = -INFINITY, L = 0.0f, acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.0f;
  merge_splits<HD>(part_o, part_ml, h, j, G, heads, base, 0, 1, n, lane, mx, L, acc);
#pragma unroll
  for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(FULL, L, o);
  store_out_row<DT, HD>(out, s, h, j, G, heads, acc, 1.0f / L, lane);
}

// Split size of a launch: 256 tokens, halved (down to 64) while the launch
// would have fewer than `target` work items and twice its splits still fit
// the workspace (cap splits); leaves the scan of the chosen size in cub/cut.
// Every CTA of both kernels runs it on the same inputs, so they agree.
__device__ __forceinline__ int pick_split(const int32_t* lens, int nseq, int heads, int64_t target, int64_t cap,
                                          int32_t* cub, int32_t* cut) {
  int split = ATT_SPLIT;
  scan_seq_lens(lens, nseq, split, cub, cut);
  while (split > 64 && (int64_t)cub[nseq] * heads < target && 2 * (int64_t)cub[nseq] <= cap) {
    split >>= 1;
    __syncthreads();  // everyone has read cub before it is rewritten
    scan_seq_lens(lens, nseq, split, cub, cut);
  }
  return split;
}

// 16-byte column `ch` of staged code row t.  SWZ = 0: rows as they lie in
// the tile.  SWZ = columns per row: XOR-swizzled so that the 8 row
// addresses of an ldmatrix (8 consecutive rows, one column) fall in 8
// different 16-byte bank groups.
template <int SWZ>
__device__ __forceinline__ int code_col(int t, int ch) {
  if (SWZ == 0) return ch;
  return SWZ >= 8 ? ch ^ (t & 7) : ch ^ (((t * SWZ) >> 3) & (SWZ - 1));
}

// Stages the raw rows of tokens tc .. tc+15 of KV head h of a quantised
// pool: at dst the 16 K code rows (row_bytes each, columns placed by
// code_col<SWZ>) then the 16 K scale/zero rows, and the same for V at dst +
// 16 x (row_bytes + meta_row_bytes).  A chunk inside one block copies its 16
// rows as they are (rows past the sequence's end included); otherwise rows
// are located one by one and rows past t_end, like those of a bad block
// (flagged), are zeros.  Commits one cp.async group.
template <int SWZ>
__device__ __forceinline__ void load_quant_chunk(uint32_t dst, const PoolGeo& g, int layer, int h,
                                                 const int32_t* btrow, int tc, int t_end, bool aligned_blocks,
                                                 int64_t vdelta, int lane, int32_t* err) {
  constexpr unsigned FULL = 0xffffffffu;
  const int RB = SWZ ? SWZ * 16 : g.row_bytes, MB = g.meta_row_bytes;
  const int RAWH = ATT_CHUNK * (RB + MB);
  const int cpr = SWZ ? SWZ : RB / 16;
  if (aligned_blocks) {
    // 16 code rows and 16 meta rows, each a contiguous run of the tile
    const int32_t blk = __ldg(btrow + tc / g.bs);
    const bool ok = blk >= 0 && blk < g.nblocks;
    if (!ok && lane == 0) atomicOr(err, DEV_ERR_BLOCK);
    const int n = ok ? 16 : 0;
    const uint8_t* tile = ok ? g.base + g.tile_off(blk, layer, 0, h) : g.base;
    const int r0 = tc % g.bs;
    const uint8_t* codes = tile + (int64_t)r0 * RB;
    const uint8_t* meta = tile + (int64_t)g.bs * RB + (int64_t)r0 * MB;
    const int cc = ATT_CHUNK * cpr, mc = ATT_CHUNK * MB / 16;
    for (int x = lane; x < cc + mc; x += 32) {
      const bool isc = x < cc;
      const int off = (isc ? x : x - cc) * 16;
      const uint8_t* sp = n ? (isc ? codes : meta) + off : g.base;
      uint32_t so;
      if (isc) {
        const int row = x / cpr;
        so = row * RB + (code_col<SWZ>(row, x - row * cpr) << 4);
      } else {
        so = ATT_CHUNK * RB + off;
      }
      cp_async16(dst + so, sp, n);
      cp_async16(dst + RAWH + so, n ? sp + vdelta : g.base, n);
    }
  } else {
    // rows from different blocks: one row's codes and meta at a time
    const int t = tc + (lane & 15);
    const uint8_t* tile = g.base;
    int nb = 0;
    if (t < t_end) {
      const int32_t blk = __ldg(btrow + t / g.bs);
      if (blk >= 0 && blk < g.nblocks) {
        tile = g.base + g.tile_off(blk, layer, 0, h);
        nb = 1;
      } else if (lane < 16) {
        atomicOr(err, DEV_ERR_BLOCK);
      }
    }
    const int rw = t % g.bs;
    const unsigned long long cp_ = reinterpret_cast<unsigned long long>(tile + (int64_t)rw * RB);
    const unsigned long long mp_ = reinterpret_cast<unsigned long long>(tile + (int64_t)g.bs * RB + (int64_t)rw * MB);
    const int mcs = MB < 16 ? MB : 16, mpr = MB / mcs;
    // each row's pointers by shuffle (all lanes), then its copies
    for (int row = 0; row < ATT_CHUNK; ++row) {
      const int ok = __shfl_sync(FULL, nb, row);
      const uint8_t* rc = reinterpret_cast<const uint8_t*>(__shfl_sync(FULL, cp_, row));
      const uint8_t* rm = reinterpret_cast<const uint8_t*>(__shfl_sync(FULL, mp_, row));
      for (int k = lane; k < cpr + mpr; k += 32) {
        if (k < cpr) {
          const uint32_t so = row * RB + (code_col<SWZ>(row, k) << 4);
          cp_async16(dst + so, ok ? rc + k * 16 : g.base, ok ? 16 : 0);
          cp_async16(dst + RAWH + so, ok ? rc + vdelta + k * 16 : g.base, ok ? 16 : 0);
        } else {
          const int m = k - cpr;
          const uint32_t so = ATT_CHUNK * RB + row * MB + m * mcs;
          const uint8_t* a = ok ? rm + m * mcs : g.base;
          const uint8_t* b = ok ? rm + vdelta + m * mcs : g.base;
          if (mcs == 16) {
            cp_async16(dst + so, a, ok ? 16 : 0);
            cp_async16(dst + RAWH + so, b, ok ? 16 : 0);
          } else if (mcs == 8) {
            cp_async8(dst + so, a, ok ? 8 : 0);
            cp_async8(dst + RAWH + so, b, ok ? 8 : 0);
          } else {
            cp_async4(dst + so, a, ok ? 4 : 0);
            cp_async4(dst + RAWH + so, b, ok ? 4 : 0);
          }
        }
      }
    }
  }
  cp_async_commit();
}

// Shared-memory layout of one stage: K rows then V rows of a 16-token chunk,
// row-major, 16-byte column chunk c of row r stored at slot c ^ (r & 7) so
// that the 8 row addresses of every ldmatrix hit 8 different bank groups.
// STAGES chunks are in flight per warp; MINB CTAs per SM; QSMEM keeps the
// queries in shared memory (same layout, 16 rows) and reads their A
// fragments with ldmatrix at every step instead of holding them in
// registers.  `split` tokens per work item (a multiple of 16).
//
// BITS = 4 or 8: a quantised pool.  A stage then holds the chunk's raw K
// code rows, K scale/zero rows, V code rows and V scale/zero rows as they
// lie in the tiles; after the wait the warp dequantises K (dq_pair, the same
// values the dequantising gather produces, rounded to the pool's type) into
// one swizzled tile in the layout above, writing zeros for rows past the
// sequence's end, computes S from it, and then dequantises V into the same
// tile for O += P V.
template <int DT, int HD, int STAGES, int MINB, bool QSMEM, int BITS = 0, bool MF32 = false>
__global__ void __launch_bounds__(ATT_WARPS * 32, MINB)
    paged_decode_attn_kernel(PoolGeo g, int layer, const uint8_t* __restrict__ q, int G,
                             const int32_t* __restrict__ bt, int bt_stride, const int32_t* __restrict__ lens,
                             int nseq, int64_t target, float scale_log2, float* __restrict__ part_o,
                             float* __restrict__ part_ml, int64_t cap_splits, uint8_t* __restrict__ out,
                             int gs_log2, unsigned long long* __restrict__ work, int32_t* err) {
  constexpr int ROWB = HD * 2;  // bytes of one K or V row (of the pool's type)
  constexpr int CPR = ROWB / 16;
  constexpr int KT = HD / 16;  // k-steps of S = Q K^T
  constexpr int NT = HD / 8;   // n-tiles of O
  constexpr unsigned FULL = 0xffffffffu;
  // stage layout: plain, K then V rows; quantised, K codes | K meta | V codes | V meta
  const int RB = g.row_bytes, MB = g.meta_row_bytes;        // code / meta row bytes
  const int RAWH = ATT_CHUNK * (RB + MB);                   // one of K, V in a quantised stage
  const int STAGE = BITS ? 2 * RAWH : 2 * ATT_CHUNK * ROWB;  // bytes per stage
  extern __shared__ __align__(128) uint8_t smem[];
  int32_t* cub = reinterpret_cast<int32_t*>(smem);
  int32_t* cut = cub + nseq + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t scan_bytes = ((size_t)2 * (nseq + 1) * 4 + 127) & ~(size_t)127;
  const int WBYTES = STAGES * STAGE + (BITS ? ATT_CHUNK * ROWB : 0) + (QSMEM ? ATT_CHUNK * ROWB : 0);
  const uint32_t wbuf = (uint32_t)__cvta_generic_to_shared(smem + scan_bytes) + warp * WBYTES;
  const uint32_t tbuf = wbuf + STAGES * STAGE;  // dequantised K, then V, of a quantised stage
  const uint32_t qbuf = tbuf + (BITS ? ATT_CHUNK * ROWB : 0);
  pdl_wait();
  pdl_release();
  const int split = pick_split(lens, nseq, g.heads, target, cap_splits, cub, cut);
  const int64_t nsplit = cub[nseq];
  if (nsplit > cap_splits) {
    if (threadIdx.x == 0) atomicOr(err, DEV_ERR_WORKSPACE);
    return;
  }
  const int64_t items = nsplit * g.heads;
  const int qheads = g.heads * G;
  // sequences of length 0 have no split: their outputs are zeros
  for (int64_t s0 = (int64_t)blockIdx.x * ATT_WARPS + warp; s0 < nseq; s0 += (int64_t)gridDim.x * ATT_WARPS)
    if (cut[s0 + 1] == cut[s0]) {
      uint4* o4 = reinterpret_cast<uint4*>(out + s0 * qheads * ROWB);
      for (int x = lane; x < qheads * CPR; x += 32) o4[x] = make_uint4(0u, 0u, 0u, 0u);
    }
  const int r = lane >> 2, c = lane & 3;
  const int64_t vdelta = (int64_t)g.heads * g.tile_bytes;  // V tile of (block, layer, head) after its K tile
  const bool aligned_blocks = (g.bs % ATT_CHUNK) == 0;     // a chunk never crosses a block
  // work items are handed out in order by a counter (zero at launch; the
  // combine kernel puts it back to zero), so warps that finish early take
  // the remaining items
  auto next_item = [&]() -> int64_t {
    unsigned long long v = 0;
    if (lane == 0) v = atomicAdd(work, 1ULL);
    return (int64_t)__shfl_sync(FULL, v, 0);
  };
  for (int64_t it = next_item(); it < items; it = next_item()) {
    const int h = (int)(it % g.heads);
    const int64_t sg = it / g.heads;
    const int s = find_seq(cub, nseq, sg);
    const int t_begin = (int)(sg - cub[s]) * split;
    const int t_end = min(cut[s + 1] - cut[s], t_begin + split);
    const int nchunks = (t_end - t_begin + ATT_CHUNK - 1) / ATT_CHUNK;
    const int32_t* btrow = bt + (int64_t)s * bt_stride;

    auto load_chunk = [&](int ci) {
      const uint32_t dst = wbuf + (ci % STAGES) * STAGE;
      const int tc = t_begin + ci * ATT_CHUNK;
      if (BITS) {
        load_quant_chunk<0>(dst, g, layer, h, btrow, tc, t_end, aligned_blocks, vdelta, lane, err);
        return;
      }
      if (aligned_blocks) {
        // the chunk's 16 rows are contiguous in one K tile (and one V tile)
        const int32_t blk = __ldg(btrow + tc / g.bs);
        const bool ok = blk >= 0 && blk < g.nblocks;
        if (!ok && lane == 0) atomicOr(err, DEV_ERR_BLOCK);
        const uint8_t* src = ok ? g.base + g.tile_off(blk, layer, 0, h) + (int64_t)(tc % g.bs) * ROWB : g.base;
#pragma unroll
        for (int i = 0; i < (ATT_CHUNK * CPR) / 32; ++i) {
          const int idx = lane + 32 * i, row = idx / CPR, ch = idx % CPR;
          const int n = (ok && tc + row < t_end) ? 16 : 0;
          const uint32_t so = row * ROWB + ((ch ^ (row & 7)) << 4);
          const uint8_t* p = n ? src + row * ROWB + ch * 16 : g.base;
          cp_async16(dst + so, p, n);
          cp_async16(dst + ATT_CHUNK * ROWB + so, n ? p + vdelta : g.base, n);
        }
      } else {
        // lanes 0..15 locate row (lane & 15); the others take it by shuffle
        const int t = tc + (lane & 15);
        const uint8_t* src = g.base;
        int nb = 0;
        if (t < t_end) {
          const int32_t blk = __ldg(btrow + t / g.bs);
          if (blk >= 0 && blk < g.nblocks) {
            src = g.base + g.tile_off(blk, layer, 0, h) + (int64_t)(t % g.bs) * ROWB;
            nb = 16;
          } else if (lane < 16) {
            atomicOr(err, DEV_ERR_BLOCK);
          }
        }
        const unsigned long long sp = reinterpret_cast<unsigned long long>(src);
#pragma unroll
        for (int i = 0; i < (ATT_CHUNK * CPR) / 32; ++i) {
          const int idx = lane + 32 * i, row = idx / CPR, ch = idx % CPR;
          const uint8_t* rp = reinterpret_cast<const uint8_t*>(__shfl_sync(FULL, sp, row));
          const int n = __shfl_sync(FULL, nb, row);
          const uint32_t so = row * ROWB + ((ch ^ (row & 7)) << 4);
          cp_async16(dst + so, n ? rp + ch * 16 : g.base, n);
          cp_async16(dst + ATT_CHUNK * ROWB + so, n ? rp + vdelta + ch * 16 : g.base, n);
        }
      }
      cp_async_commit();
    };

    float o[NT][4];
#pragma unroll
    for (int d = 0; d < NT; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // rows r and r + 8

#pragma unroll
    for (int ci = 0; ci < STAGES - 1; ++ci) {
      if (ci < nchunks) load_chunk(ci);
      else cp_async_commit();  // keep one group per slot so the wait count stays fixed
    }

    // Q as A fragments (rows = query heads, zero beyond G): in registers,
    // or staged in shared memory for ldmatrix at every step (while the
    // first chunks load).
    uint32_t qa[QSMEM ? 1 : KT][4];
    const uint8_t* qbase = q + ((int64_t)s * qheads + (int64_t)h * G) * ROWB;
    if (QSMEM) {
#pragma unroll
      for (int i = 0; i < (ATT_CHUNK * CPR) / 32; ++i) {
        const int idx = lane + 32 * i, row = idx / CPR, ch = idx % CPR;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row < G) v = __ldg(reinterpret_cast<const uint4*>(qbase + (int64_t)row * ROWB + ch * 16));
        const uint32_t a = qbuf + row * ROWB + ((ch ^ (row & 7)) << 4);
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
      }
      __syncwarp();
    } else {
#pragma unroll
      for (int kk = 0; kk < KT; ++kk)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = r + (i & 1) * 8, col = kk * 16 + 2 * c + (i >> 1) * 8;
          qa[kk][i] =
              row < G ? __ldg(reinterpret_cast<const uint32_t*>(qbase + (int64_t)row * ROWB + col * 2)) : 0u;
        }
    }

    for (int ci = 0; ci < nchunks; ++ci) {
      if (ci + STAGES - 1 < nchunks) load_chunk(ci + STAGES - 1);
      else cp_async_commit();
      cp_async_wait<STAGES - 1>();
      __syncwarp();
      const uint32_t sb = wbuf + (ci % STAGES) * STAGE;
      uint32_t kb = sb, vb = sb + ATT_CHUNK * ROWB;
      const int tc = t_begin + ci * ATT_CHUNK;
      // Quantised stage: dequantise K (then, before P V, V) into the tile;
      // rows past the end are zeros.  A task is 32 elements of one row: its
      // codes in one or two 16-byte loads, the scale/zero of its group
      // loaded once per group.
      auto dequant = [&](int kv) {
        constexpr int SPR = HD / 32;                        // 32-element segments per row
        constexpr int CBS = 32 * (BITS == 4 ? 4 : 8) / 8;  // code bytes per segment
        const int nval = min(ATT_CHUNK, t_end - tc);
#pragma unroll
        for (int i = 0; i < (ATT_CHUNK * SPR) / 32; ++i) {  // compile-time count: loads of all tasks issued together
          const int x = lane + 32 * i;
          const int seg = x % SPR, row = x / SPR;
          const uint32_t dst = tbuf + row * ROWB;
          if (row >= nval) {
#pragma unroll
            for (int k = 0; k < 4; ++k) sts128(dst + (((seg * 4 + k) ^ (row & 7)) << 4), make_uint4(0u, 0u, 0u, 0u));
            continue;
          }
          const uint32_t raw = sb + kv * RAWH;
          uint32_t cwd[8];
          {
            const uint4 a = lds128(raw + row * RB + seg * CBS);
            cwd[0] = a.x; cwd[1] = a.y; cwd[2] = a.z; cwd[3] = a.w;
            if (BITS == 8) {
              const uint4 b = lds128(raw + row * RB + seg * CBS + 16);
              cwd[4] = b.x; cwd[5] = b.y; cwd[6] = b.z; cwd[7] = b.w;
            }
          }
          const uint32_t mrow = raw + ATT_CHUNK * RB + row * MB;
          float sc = 0.0f, zr = 0.0f;
          int cur = -1;
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 8 elements per k
            const int pair = (seg * 32 + k * 8) >> gs_log2;
            if (pair != cur) {
              cur = pair;
              if (MF32) {
                const uint2 m = lds64(mrow + pair * 8);
                sc = __uint_as_float(m.x);
                zr = __uint_as_float(m.y);
              } else {
                const uint32_t m = lds32(mrow + pair * 4);
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&m));
                sc = f.x;
                zr = f.y;
              }
            }
            uint2 cw;
            uint32_t lo4 = 0, hi4 = 0;
            if (BITS == 8) {
              cw = make_uint2(cwd[2 * k], cwd[2 * k + 1]);
            } else {
              cw = make_uint2(cwd[k], 0u);
              lo4 = cw.x & 0x0F0F0F0Fu;
              hi4 = (cw.x >> 4) & 0x0F0F0F0Fu;
            }
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; e += 2) dq_pair<BITS == 4 ? 4 : 8, MF32>(cw, lo4, hi4, e, sc, zr, f[e], f[e + 1]);
            sts128(dst + (((seg * 4 + k) ^ (row & 7)) << 4),
                   make_uint4(pack2<DT>(f[0], f[1]), pack2<DT>(f[2], f[3]), pack2<DT>(f[4], f[5]), pack2<DT>(f[6], f[7])));
          }
        }
        __syncwarp();
      };
      if (BITS) {
        dequant(0);
        kb = tbuf;
      }

      // S = Q K^T: two n-tiles of 8 tokens
      float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        const int mi = lane >> 3, row = ((mi >> 1) << 3) + (lane & 7), ch = 2 * kk + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + row * ROWB + ((ch ^ (row & 7)) << 4), b0, b1, b2, b3);
        if (QSMEM) {
          // A fragment: matrices (rows 0-7 | 8-15) x (k 0-7 | 8-15) of step kk
          const int qrow = ((mi & 1) << 3) + (lane & 7), qch = 2 * kk + (mi >> 1);
          ldsm_x4(qbuf + qrow * ROWB + ((qch ^ (qrow & 7)) << 4), qa[0][0], qa[0][1], qa[0][2], qa[0][3]);
          mma16816<DT>(sacc[0], qa[0], b0, b1);
          mma16816<DT>(sacc[1], qa[0], b2, b3);
        } else {
          mma16816<DT>(sacc[0], qa[kk], b0, b1);
          mma16816<DT>(sacc[1], qa[kk], b2, b3);
        }
      }
      // online softmax (log2 domain), masking tokens past the split's end
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool valid = tc + 8 * j + 2 * c + e < t_end;
          sacc[j][e] = valid ? sacc[j][e] * scale_log2 : -INFINITY;
          sacc[j][2 + e] = valid ? sacc[j][2 + e] * scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, sacc[j][e]);
          mx1 = fmaxf(mx1, sacc[j][2 + e]);
        }
      mx0 = fmaxf(mx0, __shfl_xor_sync(FULL, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(FULL, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(FULL, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(FULL, mx1, 2));
      const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);  // finite: every chunk has a valid token
      const float a0 = ex2(m0 - n0), a1 = ex2(m1 - n1);
      m0 = n0;
      m1 = n1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          sacc[j][e] = ex2(sacc[j][e] - n0);
          sacc[j][2 + e] = ex2(sacc[j][2 + e] - n1);
          ps0 += sacc[j][e];
          ps1 += sacc[j][2 + e];
        }
      l0 = l0 * a0 + ps0;
      l1 = l1 * a1 + ps1;
      if (__any_sync(FULL, a0 != 1.0f || a1 != 1.0f)) {
#pragma unroll
        for (int d = 0; d < NT; ++d) {
          o[d][0] *= a0;
          o[d][1] *= a0;
          o[d][2] *= a1;
          o[d][3] *= a1;
        }
      }
      if (BITS) {
        __syncwarp();  // every lane has read K from the tile
        dequant(1);
        vb = tbuf;
      }
      // O += P V; P's accumulator layout is the A-fragment layout
      uint32_t pa[4];
      pa[0] = pack2<DT>(sacc[0][0], sacc[0][1]);
      pa[1] = pack2<DT>(sacc[0][2], sacc[0][3]);
      pa[2] = pack2<DT>(sacc[1][0], sacc[1][1]);
      pa[3] = pack2<DT>(sacc[1][2], sacc[1][3]);
#pragma unroll
      for (int d2 = 0; d2 < HD / 16; ++d2) {
        const int mi = lane >> 3, row = ((mi & 1) << 3) + (lane & 7), ch = 2 * d2 + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + row * ROWB + ((ch ^ (row & 7)) << 4), b0, b1, b2, b3);
        mma16816<DT>(o[2 * d2], pa, b0, b1);
        mma16816<DT>(o[2 * d2 + 1], pa, b2, b3);
      }
      __syncwarp();  // the stage is overwritten by the next load
    }
    cp_async_wait<0>();
    __syncwarp();

    l0 += __shfl_xor_sync(FULL, l0, 1);
    l0 += __shfl_xor_sync(FULL, l0, 2);
    l1 += __shfl_xor_sync(FULL, l1, 1);
    l1 += __shfl_xor_sync(FULL, l1, 2);
    const int nsp = cub[s + 1] - cub[s];
    if (nsp == 1) {  // the whole sequence in this item: normalise and write the output
      const float i0 = 1.0f / l0, i1 = 1.0f / l1;
      uint8_t* ob = out + ((int64_t)s * qheads + (int64_t)h * G) * ROWB;
#pragma unroll
      for (int d = 0; d < NT; ++d) {
        if (r < G) *reinterpret_cast<uint32_t*>(ob + r * ROWB + (8 * d + 2 * c) * 2) = pack2<DT>(o[d][0] * i0, o[d][1] * i0);
        if (r + 8 < G)
          *reinterpret_cast<uint32_t*>(ob + (r + 8) * ROWB + (8 * d + 2 * c) * 2) = pack2<DT>(o[d][2] * i1, o[d][3] * i1);
      }
      continue;
    }
    float* po = part_o + it * (int64_t)G * HD;
    float* pml = part_ml + it * (int64_t)2 * G;
#pragma unroll
    for (int d = 0; d < NT; ++d) {
      if (r < G) *reinterpret_cast<float2*>(po + r * HD + 8 * d + 2 * c) = make_float2(o[d][0], o[d][1]);
      if (r + 8 < G) *reinterpret_cast<float2*>(po + (r + 8) * HD + 8 * d + 2 * c) = make_float2(o[d][2], o[d][3]);
    }
    if (c == 0) {
      if (r < G) *reinterpret_cast<float2*>(pml + 2 * r) = make_float2(m0, l0);
      if (r + 8 < G) *reinterpret_cast<float2*>(pml + 2 * (r + 8)) = make_float2(m1, l1);
    }
  }
}

// ---------------------------------------------------------------------------
// Quantised pools read as codes (8-bit with group_size >= 16, 4-bit with
// group_size >= 32).  Instead of dequantising K and V into a tile, the warp
// feeds the tensor cores the codes themselves, as exact f16 integers built
// in registers from the staged code rows, and applies each token's
// per-group scale s and zero z around the products.  The products are
// transposed against the kernel above: tokens are the M rows and the query
// heads the N columns (G <= 8: one 8-wide n-tile; up to 16: two), so a
// 16-token chunk costs one MMA per k-step instead of two:
//   S^T = K Q^T:  S^T[t][j] = sum over groups g of
//                 s_tg (c_tg . q'_jg) + z_tg (sum of q'_jg),
//   O^T += V^T P^T:  O^T[d][j] += smax_g ((C_g^T (P^T o s_g / smax_g))[d][j]
//                                  + (sum_t P[j][t] z_tg) / smax_g)
// with q' = q / max|q| of its row in f16 (the factor returns in the softmax
// scale) and smax_g the chunk's largest |s_tg| (the f16 weights P s / smax
// stay in [-1, 1] whatever the scales).
//
// A code enters as the f16 that a byte permute (or a mask) makes of it
// directly: 1024 + code (8-bit; 4-bit low nibbles) or 64 + code (4-bit high
// nibbles, in place: ulp 1/16).  The offsets are taken out in f32 through the
// zero terms: per group, S^T gets - s (1024 sum of q' over the dims riding on
// 1024 + 64 sum over those riding on 64), and O^T's accumulator starts at
// sum_t P z / smax - (offset + 2^(bits-1)) sum_t P s / smax, with the weights
// P s / smax summed as rounded, so that the products see centred codes
// (code - 2^(bits-1)) and the zeros z + 2^(bits-1) s.  The two sums that
// span lanes -- the queries' per-group sums and the rounded weights' per-head
// sums -- are MMAs against constant A operands (all ones; the offsets), not
// shuffle reductions.
//
// Fragments come straight from the staged code rows (16-byte columns
// XOR-swizzled, read with ldmatrix):
//   * K, non-transposed: a lane receives 4 code bytes of token r (or r + 8);
//     they serve as the lane's k positions {2c, 2c+1, 2c+8, 2c+9} of one
//     k-step (8-bit) or of two k-steps (4-bit), and the queries, held as B
//     fragments in registers for the whole item, take their dimensions in
//     the same order, so the dot products are unchanged;
//   * V, transposed: a lane receives tokens (2c, 2c+1) x 2 code bytes, which
//     become A rows r and r + 8 of one m-tile (8-bit: dims 2r, 2r+1 of the
//     column) or of two (4-bit: dims 4r .. 4r+3); the output is written
//     back in dimension order;
//   * P^T o s: the S^T accumulators (token r, heads 2c, 2c+1) scaled per
//     token, packed to f16 and transposed in registers (movmatrix) into the
//     B fragments (tokens 2c, 2c+1, head r).
// A group spans whole k-steps and whole code columns, hence the floor on
// the group size; the group size is a template parameter, so every
// group boundary and meta offset is known at compile time.

// Two code bytes of w (selector 0x4j4i: bytes i, j) as the f16 pair
// (1024 + code_i, 1024 + code_j).
__device__ __forceinline__ uint32_t codes8(uint32_t w, uint32_t sel) { return __byte_perm(w, 0x64646464u, sel); }
// Eight 4-bit codes of w as four f16 pairs: low nibbles of bytes 0 and 2
// (1024 + n), high nibbles of bytes 0 and 2 (64 + n), then the same of
// bytes 1 and 3.
__device__ __forceinline__ void codes4(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t w8 = w >> 8;
  p[0] = (w & 0x000F000Fu) | 0x64006400u;
  p[1] = (w & 0x00F000F0u) | 0x54005400u;
  p[2] = (w8 & 0x000F000Fu) | 0x64006400u;
  p[3] = (w8 & 0x00F000F0u) | 0x54005400u;
}

// An 8x8 matrix of 16-bit elements held as ldmatrix holds it (lane 4i + j:
// row i, elements 2j, 2j+1), transposed.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// D = A B + C with separate C registers (f16 inputs, f32 accumulation).
__device__ __forceinline__ void mma16816_c(float* d, const uint32_t* a, uint32_t b0, uint32_t b1, float c0, float c1,
                                           float c2, float c3) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


template <int HD, int BITS, int GS, int NH, int STAGES, int MINB>
__global__ void __launch_bounds__(ATT_WARPS * 32, MINB)
    paged_decode_attn_codes_kernel(PoolGeo g, int layer, const uint8_t* __restrict__ q, int G,
                                   const int32_t* __restrict__ bt, int bt_stride, const int32_t* __restrict__ lens,
                                   int nseq, int64_t target, float scale_log2, float* __restrict__ part_o,
                                   float* __restrict__ part_ml, int64_t cap_splits, uint8_t* __restrict__ out,
                                   int gs_log2, unsigned long long* __restrict__ work, int32_t* err) {
  constexpr int ROWB = HD * 2;             // bytes of a query or output row
  constexpr int CPR = ROWB / 16;
  constexpr int RB = HD * BITS / 8;        // bytes of a code row
  constexpr int NSEG = RB / 16;            // 16-byte code columns per row
  constexpr int SEGD = 128 / BITS;         // dimensions per code column
  constexpr int KT = HD / 16;              // k-steps of S^T
  constexpr int MPS = BITS == 8 ? 1 : 2;   // m-tiles of O^T (16 dims) per code column; k-steps per column
  constexpr int MT = NSEG * MPS;           // m-tiles of O^T
  constexpr int NG = HD / GS;              // groups per row
  constexpr int CU = ATT_CHUNK * NSEG / 32;  // 16-byte code units per lane per chunk, K or V
  constexpr float OFF = (float)(1 << (BITS - 1));  // centring of the codes
  constexpr unsigned FULL = 0xffffffffu;
  static_assert(NSEG % 2 == 0 && CU >= 1 && (BITS == 8 || BITS == 4) && (NH == 1 || NH == 2), "shape");
  static_assert(GS >= 16 * MPS && GS <= HD && NG <= 8, "a group spans whole k-steps and code columns");
  const int MB = g.meta_row_bytes;
  const bool mf32 = MB == NG * 8;          // f32 (scale, zero) pairs, else f16
  const bool bf = g.dtype == RMLX_BF16;
  const int RAWH = ATT_CHUNK * (RB + MB);  // K (or V) part of a stage
  const int STAGE = 2 * RAWH;
  extern __shared__ __align__(128) uint8_t smem[];
  int32_t* cub = reinterpret_cast<int32_t*>(smem);
  int32_t* cut = cub + nseq + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t scan_bytes = ((size_t)2 * (nseq + 1) * 4 + 127) & ~(size_t)127;
  const int WBYTES = STAGES * STAGE;
  const uint32_t wbuf = (uint32_t)__cvta_generic_to_shared(smem + scan_bytes) + warp * WBYTES;
  pdl_wait();
  pdl_release();
  const int split = pick_split(lens, nseq, g.heads, target, cap_splits, cub, cut);
  const int64_t nsplit = cub[nseq];
  if (nsplit > cap_splits) {
    if (threadIdx.x == 0) atomicOr(err, DEV_ERR_WORKSPACE);
    return;
  }
  const int64_t items = nsplit * g.heads;
  const int qheads = g.heads * G;
  for (int64_t s0 = (int64_t)blockIdx.x * ATT_WARPS + warp; s0 < nseq; s0 += (int64_t)gridDim.x * ATT_WARPS)
    if (cut[s0 + 1] == cut[s0]) {
      uint4* o4 = reinterpret_cast<uint4*>(out + s0 * qheads * ROWB);
      for (int x = lane; x < qheads * CPR; x += 32) o4[x] = make_uint4(0u, 0u, 0u, 0u);
    }
  const int r = lane >> 2, c = lane & 3, mi = lane >> 3;
  const int trow = ((mi & 1) << 3) + (lane & 7);  // the token row this lane addresses in ldmatrix
  const int64_t vdelta = (int64_t)g.heads * g.tile_bytes;
  const bool aligned_blocks = (g.bs % ATT_CHUNK) == 0;
  // items handed out as in the kernel above
  auto next_item = [&]() -> int64_t {
    unsigned long long v = 0;
    if (lane == 0) v = atomicAdd(work, 1ULL);
    return (int64_t)__shfl_sync(FULL, v, 0);
  };
  for (int64_t it = next_item(); it < items; it = next_item()) {
    const int h = (int)(it % g.heads);
    const int64_t sg = it / g.heads;
    const int s = find_seq(cub, nseq, sg);
    const int t_begin = (int)(sg - cub[s]) * split;
    const int t_end = min(cut[s + 1] - cut[s], t_begin + split);
    const int nchunks = (t_end - t_begin + ATT_CHUNK - 1) / ATT_CHUNK;
    const int32_t* btrow = bt + (int64_t)s * bt_stride;

    // chunks are loaded in order: the block table entry and row of the next one
    int ld_blk = 0, ld_row = 0;
    if (aligned_blocks) {
      ld_blk = t_begin / g.bs;
      ld_row = t_begin - ld_blk * g.bs;
    }
    auto load_chunk = [&](int ci) {
      const uint32_t dst = wbuf + (ci % STAGES) * STAGE;
      if (!aligned_blocks) {
        load_quant_chunk<NSEG>(dst, g, layer, h, btrow, t_begin + ci * ATT_CHUNK, t_end, false, vdelta, lane, err);
        return;
      }
      // the chunk's 16 code rows and 16 meta rows are each a contiguous run of the tile
      const int32_t blk = __ldg(btrow + ld_blk);
      const bool ok = blk >= 0 && blk < g.nblocks;
      if (!ok && lane == 0) atomicOr(err, DEV_ERR_BLOCK);
      const int nb = ok ? 16 : 0;
      const uint8_t* tile = ok ? g.base + g.tile_off(blk, layer, 0, h) : g.base;
      const uint8_t* codes = tile + ld_row * RB;
#pragma unroll
      for (int i = 0; i < CU; ++i) {
        const int u = lane + 32 * i, row = u / NSEG, ch = u % NSEG;
        const uint32_t so = row * RB + (code_col<NSEG>(row, ch) << 4);
        const uint8_t* sp = ok ? codes + u * 16 : g.base;
        cp_async16(dst + so, sp, nb);
        cp_async16(dst + RAWH + so, ok ? sp + vdelta : g.base, nb);
      }
      const uint8_t* meta = tile + (int64_t)g.bs * RB + ld_row * MB;
      for (int x = lane; x < MB; x += 32) {  // 16 meta rows = MB 16-byte units
        const uint8_t* sp = ok ? meta + x * 16 : g.base;
        cp_async16(dst + ATT_CHUNK * RB + x * 16, sp, nb);
        cp_async16(dst + RAWH + ATT_CHUNK * RB + x * 16, ok ? sp + vdelta : g.base, nb);
      }
      cp_async_commit();
      ld_row += ATT_CHUNK;
      if (ld_row == g.bs) {
        ld_row = 0;
        ++ld_blk;
      }
    };

    float o[NH][MT][4];
#pragma unroll
    for (int n = 0; n < NH; ++n)
#pragma unroll
      for (int d = 0; d < MT; ++d) o[n][d][0] = o[n][d][1] = o[n][d][2] = o[n][d][3] = 0.0f;
    float mrun[NH][2], lrun[NH][2];  // heads 8n + 2c + e: running max, this lane's share of the sum
#pragma unroll
    for (int n = 0; n < NH; ++n) mrun[n][0] = mrun[n][1] = -INFINITY, lrun[n][0] = lrun[n][1] = 0.0f;

#pragma unroll
    for (int ci = 0; ci < STAGES - 1; ++ci) {
      if (ci < nchunks) load_chunk(ci);
      else cp_async_commit();
    }

    // Queries (while the first chunks load) as B fragments: n-tile n,
    // k-step kk holds head 8n + r at k positions (2c, 2c+1) and (2c+8,
    // 2c+9), in f16 after division by the row's max |q|.  Their sums per
    // group come from MMAs against ones, per lane for heads 8n + 2c, 2c+1
    // (the S^T columns it holds): qsx over the k positions whose codes ride
    // on 1024, qsy (4-bit) over those riding on 64.
    uint32_t qb[NH][KT][2];
    float fsc[NH][2];  // softmax scale x max|q| of heads 8n + 2c + e
    float qsx[NH][NG][2], qsy[NH][NG][2];
#pragma unroll
    for (int n = 0; n < NH; ++n) {
      const int hr = 8 * n + r;
      const uint8_t* qrow = q + ((int64_t)s * qheads + (int64_t)h * G + hr) * ROWB;
      constexpr int NW = HD / 8;  // 32-bit words (2 dims) per lane: 8-bit 16kk + 4c + (0..3); 4-bit 32j + 8c + (0..7)
      uint32_t w[NW];
      if (BITS == 8) {
#pragma unroll
        for (int kk = 0; kk < KT; ++kk) {
          const uint2 v = hr < G ? __ldg(reinterpret_cast<const uint2*>(qrow + (16 * kk + 4 * c) * 2)) : make_uint2(0u, 0u);
          w[2 * kk] = v.x;
          w[2 * kk + 1] = v.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < NSEG; ++j) {
          const uint4 v = hr < G ? __ldg(reinterpret_cast<const uint4*>(qrow + (32 * j + 8 * c) * 2)) : make_uint4(0u, 0u, 0u, 0u);
          w[(4 * j) % NW] = v.x;
          w[(4 * j + 1) % NW] = v.y;
          w[(4 * j + 2) % NW] = v.z;
          w[(4 * j + 3) % NW] = v.w;
        }
      }
      auto unpack = [&](uint32_t x) -> float2 {
        if (bf) return make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xffff0000u));
        return __half22float2(*reinterpret_cast<const __half2*>(&x));
      };
      float mx = 0.0f;
#pragma unroll
      for (int i = 0; i < NW; ++i) {
        const float2 t2 = unpack(w[i]);
        mx = fmaxf(mx, fmaxf(fabsf(t2.x), fabsf(t2.y)));
      }
      mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 2));
      const float msc = mx > 0.0f ? mx : 1.0f, inv = rcp_approx(msc);
#pragma unroll
      for (int i = 0; i < NW; ++i) {
        const float2 t2 = unpack(w[i]);
        w[i] = pack2<RMLX_F16>(t2.x * inv, t2.y * inv);
      }
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        if (BITS == 8) {  // k-step kk: dims 16kk + 4c + (0, 1) | (2, 3)
          qb[n][kk][0] = w[2 * kk];
          qb[n][kk][1] = w[2 * kk + 1];
        } else {  // k-step 2j + u: dims 32j + 8c + (2u, 2u+4) | (2u+1, 2u+5)
          const int j = kk >> 1, u = kk & 1;
          qb[n][kk][0] = __byte_perm(w[(4 * j + u) % NW], w[(4 * j + 2 + u) % NW], 0x5410);
          qb[n][kk][1] = __byte_perm(w[(4 * j + u) % NW], w[(4 * j + 2 + u) % NW], 0x7632);
        }
      }
      constexpr uint32_t ONE2 = 0x3C003C00u;  // (1.0, 1.0) in f16
      const uint32_t ax[4] = {ONE2, ONE2, BITS == 8 ? ONE2 : 0u, BITS == 8 ? ONE2 : 0u};
      const uint32_t ay[4] = {0u, 0u, ONE2, ONE2};
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) {
        float dx[4] = {0.f, 0.f, 0.f, 0.f}, dy[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < GS / 16; ++k) {
          const int kk = gg * (GS / 16) + k;
          mma16816<RMLX_F16>(dx, ax, qb[n][kk][0], qb[n][kk][1]);
          if (BITS == 4) mma16816<RMLX_F16>(dy, ay, qb[n][kk][0], qb[n][kk][1]);
        }
        qsx[n][gg][0] = dx[0];
        qsx[n][gg][1] = dx[1];
        qsy[n][gg][0] = dy[0];
        qsy[n][gg][1] = dy[1];
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) fsc[n][e] = __shfl_sync(FULL, msc, (2 * c + e) * 4) * scale_log2;
    }

    for (int ci = 0; ci < nchunks; ++ci) {
      if (ci + STAGES - 1 < nchunks) load_chunk(ci + STAGES - 1);
      else cp_async_commit();
      cp_async_wait<STAGES - 1>();
      __syncwarp();
      const uint32_t kraw = wbuf + (ci % STAGES) * STAGE, vraw = kraw + RAWH;
      const uint32_t kmeta = kraw + ATT_CHUNK * RB, vmeta = vraw + ATT_CHUNK * RB;
      const int nval = min(ATT_CHUNK, t_end - t_begin - ci * ATT_CHUNK);
      const bool val0 = r < nval, val1 = r + 8 < nval;  // this lane's tokens r and r + 8
      // (scale, zero) of group gi for tokens r and r + 8; zeros past the end
      auto load_meta = [&](uint32_t mbase, int gi, float& s0, float& z0, float& s1, float& z1) {
        float a[2], b[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint32_t ad = mbase + (r + 8 * k) * MB;
          if (mf32) {
            const uint2 m = lds64(ad + gi * 8);
            a[k] = __uint_as_float(m.x);
            b[k] = __uint_as_float(m.y);
          } else {
            const uint32_t m = lds32(ad + gi * 4);
            const float2 fm = __half22float2(*reinterpret_cast<const __half2*>(&m));
            a[k] = fm.x;
            b[k] = fm.y;
          }
        }
        s0 = val0 ? a[0] : 0.0f;
        z0 = val0 ? b[0] : 0.0f;
        s1 = val1 ? a[1] : 0.0f;
        z1 = val1 ? b[1] : 0.0f;
      };

      // S^T = K Q^T, folded into sacc at the end of each group
      // a group's products; 4-bit: even k-steps in sgp, odd in sgq (two
      // shorter MMA chains; measured 86.6 against 88.5 us per layer, while
      // 8-bit pools measured no gain)
      float sacc[NH][4], sgp[NH][4], sgq[NH][4];
#pragma unroll
      for (int n = 0; n < NH; ++n)
#pragma unroll
        for (int k = 0; k < 4; ++k) sacc[n][k] = sgp[n][k] = sgq[n][k] = 0.0f;
#pragma unroll
      for (int sc2 = 0; sc2 < NSEG; sc2 += 2) {
        uint32_t wv[4];  // tokens 0-7 | 8-15 of column sc2, then of column sc2 + 1
        ldsm_x4(kraw + trow * RB + (code_col<NSEG>(trow, sc2 + (mi >> 1)) << 4), wv[0], wv[1], wv[2], wv[3]);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t lo = wv[2 * half], hi = wv[2 * half + 1];  // tokens r, r + 8
          uint32_t a[MPS][4];
          if (BITS == 8) {
            a[0][0] = codes8(lo, 0x4140u);
            a[0][1] = codes8(hi, 0x4140u);
            a[0][2] = codes8(lo, 0x4342u);
            a[0][3] = codes8(hi, 0x4342u);
          } else {
            uint32_t pl[4], ph[4];
            codes4(lo, pl);
            codes4(hi, ph);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              a[u][0] = pl[2 * u];
              a[u][1] = ph[2 * u];
              a[u][2] = pl[2 * u + 1];
              a[u][3] = ph[2 * u + 1];
            }
          }
#pragma unroll
          for (int u = 0; u < MPS; ++u) {
            const int kk = (sc2 + half) * MPS + u;
#pragma unroll
            for (int n = 0; n < NH; ++n)
              mma16816<RMLX_F16>((BITS == 4 && (kk & 1)) ? sgq[n] : sgp[n], a[u], qb[n][kk][0], qb[n][kk][1]);
            if (((kk + 1) * 16) % GS == 0) {  // the group ends with this k-step
              const int gk = kk * 16 / GS;
              float s0, z0, s1, z1;
              load_meta(kmeta, gk, s0, z0, s1, z1);
              // zeros net of the offsets: x sums ride on 1024, y sums on 64
              const float zx0 = fmaf(s0, -1024.0f, z0), zx1 = fmaf(s1, -1024.0f, z1);
              const float zy0 = fmaf(s0, -64.0f, z0), zy1 = fmaf(s1, -64.0f, z1);
#pragma unroll
              for (int n = 0; n < NH; ++n) {
                const float* qx = qsx[n][gk];
                const float* qy = qsy[n][gk];
                if (BITS == 4) {
#pragma unroll
                  for (int k = 0; k < 4; ++k) sgp[n][k] += sgq[n][k];
                }
                float t[4] = {fmaf(s0, sgp[n][0], zx0 * qx[0]), fmaf(s0, sgp[n][1], zx0 * qx[1]),
                              fmaf(s1, sgp[n][2], zx1 * qx[0]), fmaf(s1, sgp[n][3], zx1 * qx[1])};
                if (BITS == 4) {
                  t[0] = fmaf(zy0, qy[0], t[0]);
                  t[1] = fmaf(zy0, qy[1], t[1]);
                  t[2] = fmaf(zy1, qy[0], t[2]);
                  t[3] = fmaf(zy1, qy[1], t[3]);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  sacc[n][k] += t[k];
                  sgp[n][k] = sgq[n][k] = 0.0f;
                }
              }
            }
          }
        }
      }
      // online softmax (log2 domain) per head over the chunk's tokens
      bool rescale = false;
      float al[NH][2];
#pragma unroll
      for (int n = 0; n < NH; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float x0 = val0 ? sacc[n][e] * fsc[n][e] : -INFINITY;
          const float x1 = val1 ? sacc[n][2 + e] * fsc[n][e] : -INFINITY;
          float mx = fmaxf(x0, x1);
          mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 16));
          const float nm = fmaxf(mrun[n][e], mx);  // finite: every chunk has a valid token
          al[n][e] = ex2(mrun[n][e] - nm);
          mrun[n][e] = nm;
          sacc[n][e] = ex2(x0 - nm);
          sacc[n][2 + e] = ex2(x1 - nm);
          lrun[n][e] = lrun[n][e] * al[n][e] + (sacc[n][e] + sacc[n][2 + e]);
          rescale |= al[n][e] != 1.0f;
        }
      if (__any_sync(FULL, rescale)) {
#pragma unroll
        for (int n = 0; n < NH; ++n)
#pragma unroll
          for (int d = 0; d < MT; ++d) {
            o[n][d][0] *= al[n][0];
            o[n][d][1] *= al[n][1];
            o[n][d][2] *= al[n][0];
            o[n][d][3] *= al[n][1];
          }
      }

      // O^T += V^T P^T, one group at a time
      uint32_t pb[NH][2];
      float cz[NH][4], smx = 1.0f;
#pragma unroll
      for (int sc2 = 0; sc2 < NSEG; sc2 += 2) {
        uint32_t wv[4];  // tokens (2c, 2c+1) | (8+2c, 9+2c) of column sc2, then of column sc2 + 1
        ldsm_x4_t(vraw + trow * RB + (code_col<NSEG>(trow, sc2 + (mi >> 1)) << 4), wv[0], wv[1], wv[2], wv[3]);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int col = sc2 + half;
          if ((col * SEGD) % GS == 0) {  // the column starts a group
            const int gv = col * SEGD / GS;
            float s0, z0, s1, z1;
            load_meta(vmeta, gv, s0, z0, s1, z1);
            float am = fmaxf(fabsf(s0), fabsf(s1));
            am = fmaxf(am, __shfl_xor_sync(FULL, am, 4));
            am = fmaxf(am, __shfl_xor_sync(FULL, am, 8));
            am = fmaxf(am, __shfl_xor_sync(FULL, am, 16));
            smx = am > 0.0f ? am : 1.0f;
            const float inv = rcp_approx(smx), a0 = s0 * inv, a1 = s1 * inv;
            const float zc0 = fmaf(s0, OFF, z0) * inv, zc1 = fmaf(s1, OFF, z1) * inv;  // centred zeros / smax
            // A of the offsets' MMA: rows r and r + 8 hold -(offset + 2^(bits-1)) for codes
            // on 1024 (8-bit, 4-bit low nibbles: -1152, -1032) or on 64 (4-bit high nibbles: -72)
            const uint32_t ar = BITS == 8 ? 0xE480E480u : 0xE408E408u, ar8 = BITS == 8 ? 0xE480E480u : 0xD480D480u;
            const uint32_t aoff[4] = {ar, ar8, ar, ar8};
#pragma unroll
            for (int n = 0; n < NH; ++n) {
              pb[n][0] = movmatrix_t(pack2<RMLX_F16>(sacc[n][0] * a0, sacc[n][1] * a0));
              pb[n][1] = movmatrix_t(pack2<RMLX_F16>(sacc[n][2] * a1, sacc[n][3] * a1));
              // per head: sum_t P z' / smax ...
              float zs[2] = {fmaf(sacc[n][0], zc0, sacc[n][2] * zc1), fmaf(sacc[n][1], zc0, sacc[n][3] * zc1)};
#pragma unroll
              for (int e = 0; e < 2; ++e) {
#pragma unroll
                for (int o2 = 4; o2 < 32; o2 <<= 1) zs[e] += __shfl_xor_sync(FULL, zs[e], o2);
              }
              // ... less the offsets times the sum of the rounded weights
              mma16816_c(cz[n], aoff, pb[n][0], pb[n][1], zs[0], zs[1], zs[0], zs[1]);
            }
          }
          const uint32_t lo = wv[2 * half], hi = wv[2 * half + 1];
          uint32_t a[MPS][4];
          if (BITS == 8) {  // rows r, r + 8: dims 2r, 2r + 1 of the column
            a[0][0] = codes8(lo, 0x4240u);
            a[0][1] = codes8(lo, 0x4341u);
            a[0][2] = codes8(hi, 0x4240u);
            a[0][3] = codes8(hi, 0x4341u);
          } else {  // m-tile u, rows r, r + 8: dims 4r + 2u, 4r + 2u + 1 of the column
            uint32_t pl[4], ph[4];
            codes4(lo, pl);
            codes4(hi, ph);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              a[u][0] = pl[2 * u];
              a[u][1] = pl[2 * u + 1];
              a[u][2] = ph[2 * u];
              a[u][3] = ph[2 * u + 1];
            }
          }
#pragma unroll
          for (int u = 0; u < MPS; ++u)
#pragma unroll
            for (int n = 0; n < NH; ++n) {
              float t[4];
              mma16816_c(t, a[u], pb[n][0], pb[n][1], cz[n][0], cz[n][1], cz[n][2], cz[n][3]);
              float* od = o[n][col * MPS + u];
              od[0] = fmaf(smx, t[0], od[0]);
              od[1] = fmaf(smx, t[1], od[1]);
              od[2] = fmaf(smx, t[2], od[2]);
              od[3] = fmaf(smx, t[3], od[3]);
            }
        }
      }
      __syncwarp();  // the stage is overwritten by the next load
    }
    cp_async_wait<0>();
    __syncwarp();

    // m-tile col * MPS + u, rows r and r + 8 hold dimensions
    // col * SEGD + 2 MPS r + 2u and + 1; elements e, 2 + e head 8n + 2c + e
    const int nsp = cub[s + 1] - cub[s];
#pragma unroll
    for (int n = 0; n < NH; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float lt = lrun[n][e];
        lt += __shfl_xor_sync(FULL, lt, 4);
        lt += __shfl_xor_sync(FULL, lt, 8);
        lt += __shfl_xor_sync(FULL, lt, 16);
        const int hq = 8 * n + 2 * c + e;  // query head within the group
        if (hq >= G) continue;
        if (nsp == 1) {
          const float il = 1.0f / lt;
          uint8_t* ob = out + ((int64_t)s * qheads + (int64_t)h * G + hq) * ROWB;
#pragma unroll
          for (int col = 0; col < NSEG; ++col) {
            const int d0 = col * SEGD + 2 * MPS * r;
            uint32_t w[MPS];
#pragma unroll
            for (int u = 0; u < MPS; ++u) {
              const float v0 = o[n][col * MPS + u][e] * il, v1 = o[n][col * MPS + u][2 + e] * il;
              w[u] = bf ? pack2<RMLX_BF16>(v0, v1) : pack2<RMLX_F16>(v0, v1);
            }
            if constexpr (MPS == 1) *reinterpret_cast<uint32_t*>(ob + d0 * 2) = w[0];
            else *reinterpret_cast<uint2*>(ob + d0 * 2) = make_uint2(w[0], w[1]);
          }
        } else {
          float* po = part_o + (it * (int64_t)G + hq) * HD;
#pragma unroll
          for (int col = 0; col < NSEG; ++col) {
            const int d0 = col * SEGD + 2 * MPS * r;
            if constexpr (MPS == 1) {
              *reinterpret_cast<float2*>(po + d0) = make_float2(o[n][col][e], o[n][col][2 + e]);
            } else {
              *reinterpret_cast<float4*>(po + d0) = make_float4(o[n][2 * col][e], o[n][2 * col][2 + e],
                                                                o[n][2 * col + 1][e], o[n][2 * col + 1][2 + e]);
            }
          }
          if (r == 0) *reinterpret_cast<float2*>(part_ml + it * (int64_t)2 * G + 2 * hq) = make_float2(mrun[n][e], lt);
        }
      }
  }
}

// ---------------------------------------------------------------------------
// bf16/f16 pools, with the products transposed as in the codes kernel:
// tokens are the M rows and the query heads the N columns (one 8-wide
// n-tile for G <= 8, two up to 16).  Per 16-token chunk and k-step one
// ldmatrix gives the K rows as an A fragment (no conversion), the queries
// stay in registers as B fragments for the whole item, P^T reaches the B
// operand of O^T += V^T P^T through movmatrix, and ldmatrix.trans gives V^T.
// Against the kernel above: half the MMAs, half the O registers, no query
// tile in shared memory, so three CTAs of four warps fit an SM (16 KiB of
// stages per warp).
template <int DT, int HD, int NH, int STAGES, int MINB>
__global__ void __launch_bounds__(ATT_WARPS * 32, MINB)
    paged_decode_attn_rows_kernel(PoolGeo g, int layer, const uint8_t* __restrict__ q, int G,
                                  const int32_t* __restrict__ bt, int bt_stride, const int32_t* __restrict__ lens,
                                  int nseq, int64_t target, float scale_log2, float* __restrict__ part_o,
                                  float* __restrict__ part_ml, int64_t cap_splits, uint8_t* __restrict__ out,
                                  int gs_log2, unsigned long long* __restrict__ work, int32_t* err) {
  constexpr int ROWB = HD * 2;  // bytes of a K, V, query or output row
  constexpr int CPR = ROWB / 16;
  constexpr int KT = HD / 16;   // k-steps of S^T, and m-tiles of O^T
  constexpr int STAGE = 2 * ATT_CHUNK * ROWB;  // K rows then V rows, 16-byte columns XOR-swizzled
  constexpr unsigned FULL = 0xffffffffu;
  static_assert(CPR >= 8 && (NH == 1 || NH == 2), "shape");
  extern __shared__ __align__(128) uint8_t smem[];
  int32_t* cub = reinterpret_cast<int32_t*>(smem);
  int32_t* cut = cub + nseq + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t scan_bytes = ((size_t)2 * (nseq + 1) * 4 + 127) & ~(size_t)127;
  const uint32_t wbuf = (uint32_t)__cvta_generic_to_shared(smem + scan_bytes) + warp * STAGES * STAGE;
  pdl_wait();
  pdl_release();
  const int split = pick_split(lens, nseq, g.heads, target, cap_splits, cub, cut);
  const int64_t nsplit = cub[nseq];
  if (nsplit > cap_splits) {
    if (threadIdx.x == 0) atomicOr(err, DEV_ERR_WORKSPACE);
    return;
  }
  const int64_t items = nsplit * g.heads;
  const int qheads = g.heads * G;
  for (int64_t s0 = (int64_t)blockIdx.x * ATT_WARPS + warp; s0 < nseq; s0 += (int64_t)gridDim.x * ATT_WARPS)
    if (cut[s0 + 1] == cut[s0]) {
      uint4* o4 = reinterpret_cast<uint4*>(out + s0 * qheads * ROWB);
      for (int x = lane; x < qheads * CPR; x += 32) o4[x] = make_uint4(0u, 0u, 0u, 0u);
    }
  const int r = lane >> 2, c = lane & 3, mi = lane >> 3;
  // ldmatrix row addresses: K (A of S^T) takes matrices (tokens 0-7 | 8-15) x
  // (k 0-7 | 8-15); V^T (A of O^T) takes (dims 0-7 | 8-15) x (tokens 0-7 | 8-15)
  const int krow = ((mi & 1) << 3) + (lane & 7), kcol = mi >> 1;
  const int vrow = ((mi >> 1) << 3) + (lane & 7), vcol = mi & 1;
  const int64_t vdelta = (int64_t)g.heads * g.tile_bytes;
  const bool aligned_blocks = (g.bs % ATT_CHUNK) == 0;
  auto next_item = [&]() -> int64_t {
    unsigned long long v = 0;
    if (lane == 0) v = atomicAdd(work, 1ULL);
    return (int64_t)__shfl_sync(FULL, v, 0);
  };
  for (int64_t it = next_item(); it < items; it = next_item()) {
    const int h = (int)(it % g.heads);
    const int64_t sg = it / g.heads;
    const int s = find_seq(cub, nseq, sg);
    const int t_begin = (int)(sg - cub[s]) * split;
    const int t_end = min(cut[s + 1] - cut[s], t_begin + split);
    const int nchunks = (t_end - t_begin + ATT_CHUNK - 1) / ATT_CHUNK;
    const int32_t* btrow = bt + (int64_t)s * bt_stride;

    int ld_blk = 0, ld_row = 0;  // chunks load in order: the block table entry and row of the next one
    if (aligned_blocks) {
      ld_blk = t_begin / g.bs;
      ld_row = t_begin - ld_blk * g.bs;
    }
    auto load_chunk = [&](int ci) {
      const uint32_t dst = wbuf + (ci % STAGES) * STAGE;
      if (aligned_blocks) {
        // the chunk's 16 rows are contiguous in one K tile (and one V tile)
        const int tc = t_begin + ci * ATT_CHUNK;
        const int32_t blk = __ldg(btrow + ld_blk);
        const bool ok = blk >= 0 && blk < g.nblocks;
        if (!ok && lane == 0) atomicOr(err, DEV_ERR_BLOCK);
        const uint8_t* src = ok ? g.base + g.tile_off(blk, layer, 0, h) + (int64_t)ld_row * ROWB : g.base;
#pragma unroll
        for (int i = 0; i < (ATT_CHUNK * CPR) / 32; ++i) {
          const int idx = lane + 32 * i, row = idx / CPR, ch = idx % CPR;
          const int n = (ok && tc + row < t_end) ? 16 : 0;
          const uint32_t so = row * ROWB + ((ch ^ (row & 7)) << 4);
          const uint8_t* p = n ? src + row * ROWB + ch * 16 : g.base;
          cp_async16(dst + so, p, n);
          cp_async16(dst + ATT_CHUNK * ROWB + so, n ? p + vdelta : g.base, n);
        }
        ld_row += ATT_CHUNK;
        if (ld_row == g.bs) {
          ld_row = 0;
          ++ld_blk;
        }
      } else {
        // lanes 0..15 locate row (lane & 15); the others take it by shuffle
        const int t = t_begin + ci * ATT_CHUNK + (lane & 15);
        const uint8_t* src = g.base;
        int nb = 0;
        if (t < t_end) {
          const int32_t blk = __ldg(btrow + t / g.bs);
          if (blk >= 0 && blk < g.nblocks) {
            src = g.base + g.tile_off(blk, layer, 0, h) + (int64_t)(t % g.bs) * ROWB;
            nb = 16;
          } else if (lane < 16) {
            atomicOr(err, DEV_ERR_BLOCK);
          }
        }
        const unsigned long long sp = reinterpret_cast<unsigned long long>(src);
#pragma unroll
        for (int i = 0; i < (ATT_CHUNK * CPR) / 32; ++i) {
          const int idx = lane + 32 * i, row = idx / CPR, ch = idx % CPR;
          const uint8_t* rp = reinterpret_cast<const uint8_t*>(__shfl_sync(FULL, sp, row));
          const int n = __shfl_sync(FULL, nb, row);
          const uint32_t so = row * ROWB + ((ch ^ (row & 7)) << 4);
          cp_async16(dst + so, n ? rp + ch * 16 : g.base, n);
          cp_async16(dst + ATT_CHUNK * ROWB + so, n ? rp + vdelta + ch * 16 : g.base, n);
        }
      }
      cp_async_commit();
    };

    float o[NH][KT][4];  // O^T: m-tile mt, rows r and r + 8 = dims 16 mt + r, + 8; columns heads 8n + 2c, + 1
#pragma unroll
    for (int n = 0; n < NH; ++n)
#pragma unroll
      for (int d = 0; d < KT; ++d) o[n][d][0] = o[n][d][1] = o[n][d][2] = o[n][d][3] = 0.0f;
    float mrun[NH][2], lrun[NH][2];  // heads 8n + 2c + e: running max, this lane's share of the sum
#pragma unroll
    for (int n = 0; n < NH; ++n) mrun[n][0] = mrun[n][1] = -INFINITY, lrun[n][0] = lrun[n][1] = 0.0f;

#pragma unroll
    for (int ci = 0; ci < STAGES - 1; ++ci) {
      if (ci < nchunks) load_chunk(ci);
      else cp_async_commit();
    }

    // queries as B fragments (while the first chunks load): n-tile n, k-step
    // kk holds head 8n + r at dims 16kk + 2c, +1 and 16kk + 8 + 2c, +1
    uint32_t qb[NH][KT][2];
#pragma unroll
    for (int n = 0; n < NH; ++n) {
      const int hr = 8 * n + r;
      const uint8_t* qrow = q + ((int64_t)s * qheads + (int64_t)h * G + hr) * ROWB;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        qb[n][kk][0] = hr < G ? __ldg(reinterpret_cast<const uint32_t*>(qrow + (16 * kk + 2 * c) * 2)) : 0u;
        qb[n][kk][1] = hr < G ? __ldg(reinterpret_cast<const uint32_t*>(qrow + (16 * kk + 8 + 2 * c) * 2)) : 0u;
      }
    }

    for (int ci = 0; ci < nchunks; ++ci) {
      if (ci + STAGES - 1 < nchunks) load_chunk(ci + STAGES - 1);
      else cp_async_commit();
      cp_async_wait<STAGES - 1>();
      __syncwarp();
      const uint32_t kb = wbuf + (ci % STAGES) * STAGE, vb = kb + ATT_CHUNK * ROWB;
      const int nval = min(ATT_CHUNK, t_end - t_begin - ci * ATT_CHUNK);
      const bool val0 = r < nval, val1 = r + 8 < nval;  // this lane's tokens r and r + 8

      // S^T = K Q^T
      float sacc[NH][4];
#pragma unroll
      for (int n = 0; n < NH; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        uint32_t a[4];
        const int ch = 2 * kk + kcol;
        ldsm_x4(kb + krow * ROWB + ((ch ^ (krow & 7)) << 4), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int n = 0; n < NH; ++n) mma16816<DT>(sacc[n], a, qb[n][kk][0], qb[n][kk][1]);
      }
      // online softmax (log2 domain) per head over the chunk's tokens
      bool rescale = false;
      float al[NH][2];
#pragma unroll
      for (int n = 0; n < NH; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float x0 = val0 ? sacc[n][e] * scale_log2 : -INFINITY;
          const float x1 = val1 ? sacc[n][2 + e] * scale_log2 : -INFINITY;
          float mx = fmaxf(x0, x1);
          mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 16));
          const float nm = fmaxf(mrun[n][e], mx);  // finite: every chunk has a valid token
          al[n][e] = ex2(mrun[n][e] - nm);
          mrun[n][e] = nm;
          sacc[n][e] = ex2(x0 - nm);
          sacc[n][2 + e] = ex2(x1 - nm);
          lrun[n][e] = lrun[n][e] * al[n][e] + (sacc[n][e] + sacc[n][2 + e]);
          rescale |= al[n][e] != 1.0f;
        }
      if (__any_sync(FULL, rescale)) {
#pragma unroll
        for (int n = 0; n < NH; ++n)
#pragma unroll
          for (int d = 0; d < KT; ++d) {
            o[n][d][0] *= al[n][0];
            o[n][d][1] *= al[n][1];
            o[n][d][2] *= al[n][0];
            o[n][d][3] *= al[n][1];
          }
      }
      // O^T += V^T P^T: P (rounded to the pool's type) transposed in registers
      uint32_t pb[NH][2];
#pragma unroll
      for (int n = 0; n < NH; ++n) {
        pb[n][0] = movmatrix_t(pack2<DT>(sacc[n][0], sacc[n][1]));
        pb[n][1] = movmatrix_t(pack2<DT>(sacc[n][2], sacc[n][3]));
      }
#pragma unroll
      for (int mt = 0; mt < KT; ++mt) {
        uint32_t a[4];
        const int ch = 2 * mt + vcol;
        ldsm_x4_t(vb + vrow * ROWB + ((ch ^ (vrow & 7)) << 4), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int n = 0; n < NH; ++n) mma16816<DT>(o[n][mt], a, pb[n][0], pb[n][1]);
      }
      __syncwarp();  // the stage is overwritten by the next load
    }
    cp_async_wait<0>();
    __syncwarp();

    const int nsp = cub[s + 1] - cub[s];
#pragma unroll
    for (int n = 0; n < NH; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float lt = lrun[n][e];
        lt += __shfl_xor_sync(FULL, lt, 4);
        lt += __shfl_xor_sync(FULL, lt, 8);
        lt += __shfl_xor_sync(FULL, lt, 16);
        const int hq = 8 * n + 2 * c + e;  // query head within the group
        if (hq >= G) continue;
        if (nsp == 1) {
          const float il = 1.0f / lt;
          uint8_t* ob = out + ((int64_t)s * qheads + (int64_t)h * G + hq) * ROWB;
#pragma unroll
          for (int mt = 0; mt < KT; ++mt) {
            const uint32_t w = pack2<DT>(o[n][mt][e] * il, o[n][mt][2 + e] * il);
            *reinterpret_cast<uint16_t*>(ob + (16 * mt + r) * 2) = (uint16_t)(w & 0xffffu);
            *reinterpret_cast<uint16_t*>(ob + (16 * mt + 8 + r) * 2) = (uint16_t)(w >> 16);
          }
        } else {
          float* po = part_o + (it * (int64_t)G + hq) * HD;
#pragma unroll
          for (int mt = 0; mt < KT; ++mt) {
            po[16 * mt + r] = o[n][mt][e];
            po[16 * mt + 8 + r] = o[n][mt][2 + e];
          }
          if (r == 0) *reinterpret_cast<float2*>(part_ml + it * (int64_t)2 * G + 2 * hq) = make_float2(mrun[n][e], lt);
        }
      }
  }
}

// One warp per (sequence, query head) of the sequences held by two or more
// splits (the split kernel wrote the others): combine_splits.
template <int DT, int HD>
__global__ void __launch_bounds__(256) attn_combine_kernel(const int32_t* __restrict__ lens, int nseq, int64_t target,
                                                           int heads, int G, const float* __restrict__ part_o,
                                                           const float* __restrict__ part_ml, uint8_t* __restrict__ out,
                                                           int64_t cap_splits, unsigned long long* __restrict__ work) {
  extern __shared__ int32_t cs[];
  int32_t* cub = cs;
  int32_t* cut = cs + nseq + 1;
  // seq_lens is an input of the split kernel, not one of its outputs: the
  // scan may run while that kernel drains; the partials are read after the wait
  pdl_release();
  pick_split(lens, nseq, heads, target, cap_splits, cub, cut);
  pdl_wait();
  if (blockIdx.x == 0 && threadIdx.x == 0) *work = 0;  // the split kernel has taken all its items
  if (cub[nseq] > cap_splits) return;  // flagged by the split kernel
  const int lane = threadIdx.x & 31;
  const int qheads = heads * G;
  const int64_t total = (int64_t)nseq * qheads;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total; w += nwarps) {
    const int s = (int)(w / qheads), qh = (int)(w % qheads);
    const int n = cub[s + 1] - cub[s];
    if (n < 2) continue;
    combine_splits<DT, HD>(part_o, part_ml, out, s, qh / G, qh % G, G, heads, cub[s], n, lane);
  }
}

// The same combine for launches with few (sequence, query head) pairs and
// many splits each (a KV-head shard of a few heads): one CTA per pair, its
// 8 warps merging every 8th split each (one memory round trip for up to 128
// splits), then the 8 partial (max, sum, output) in shared memory merged by
// warp 0.
template <int DT, int HD>
__global__ void __launch_bounds__(256) attn_combine_cta_kernel(const int32_t* __restrict__ lens, int nseq,
                                                               int64_t target, int heads, int G,
                                                               const float* __restrict__ part_o,
                                                               const float* __restrict__ part_ml,
                                                               uint8_t* __restrict__ out, int64_t cap_splits,
                                                               unsigned long long* __restrict__ work) {
  constexpr int EPL = HD / 32, NW = 8;
  constexpr unsigned FULL = 0xffffffffu;
  extern __shared__ int32_t cs[];
  int32_t* cub = cs;
  int32_t* cut = cs + nseq + 1;
  float* red = reinterpret_cast<float*>(cs + ((2 * (nseq + 1) + 3) & ~3));  // [NW][2 + HD]: max, sum, output
  pdl_release();
  pick_split(lens, nseq, heads, target, cap_splits, cub, cut);
  pdl_wait();
  if (blockIdx.x == 0 && threadIdx.x == 0) *work = 0;  // the split kernel has taken all its items
  if (cub[nseq] > cap_splits) return;  // flagged by the split kernel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qheads = heads * G;
  const int64_t total = (int64_t)nseq * qheads;
  for (int64_t pr = blockIdx.x; pr < total; pr += gridDim.x) {
    const int s = (int)(pr / qheads), qh = (int)(pr % qheads);
    const int n = cub[s + 1] - cub[s];
    if (n < 2) continue;  // the split kernel wrote it
    const int h = qh / G, j = qh % G;
    float mx = -INFINITY, L = 0.0f, acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.0f;
    const int nk = warp < n ? (n - warp + NW - 1) / NW : 0;
    merge_splits<HD>(part_o, part_ml, h, j, G, heads, cub[s], warp, NW, nk, lane, mx, L, acc);
#pragma unroll
    for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(FULL, L, o);
    float* rw = red + warp * (2 + HD);
    if (lane == 0) {
      rw[0] = mx;
      rw[1] = L;
    }
#pragma unroll
    for (int e = 0; e < EPL; ++e) rw[2 + lane * EPL + e] = acc[e];
    __syncthreads();
    if (warp == 0) {
      float m = -INFINITY;
#pragma unroll
      for (int w = 0; w < NW; ++w) m = fmaxf(m, red[w * (2 + HD)]);  // finite: n >= 2 splits
      float lt = 0.0f, o[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[e] = 0.0f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float* r = red + w * (2 + HD);
        const float a = ex2(r[0] - m);  // 0 for a warp without splits (max -inf)
        lt += a * r[1];
#pragma unroll
        for (int e = 0; e < EPL; ++e) o[e] += a * r[2 + lane * EPL + e];
      }
      store_out_row<DT, HD>(out, s, h, j, G, heads, o, 1.0f / lt, lane);
    }
    __syncthreads();  // red is reused by the next pair
  }
}

}  // namespace rmlx

using namespace rmlx;

namespace {

// Bytes of workspace per split and KV head: G x head_dim partial outputs and
// a (max, sum) pair per query head, all f32.
size_t split_bytes(int heads, int G, int hd) { return (size_t)heads * G * (hd + 2) * sizeof(float); }

using AttnFn = void (*)(PoolGeo, int, const uint8_t*, int, const int32_t*, int, const int32_t*, int, int64_t,
                        float, float*, float*, int64_t, uint8_t*, int, unsigned long long*, int32_t*);
using CombineFn = void (*)(const int32_t*, int, int64_t, int, int, const float*, const float*, uint8_t*, int64_t,
                           unsigned long long*);

// Work items a launch wants before it halves its split size: items_x2 / 2
// per resident warp.  Fewer, longer items save per-item work (queries,
// partials, combine); more items even out the tail.  Measured per kernel:
// 1 for the bf16/f16 and 8-bit codes kernels, 3 for the 4-bit one.
int64_t attn_target(AttnFn fa, size_t smem, int num_sms, int items_x2) {
  return (int64_t)items_x2 * persistent_grid(fa, ATT_WARPS * 32, smem, num_sms) * ATT_WARPS / 2;
}

// The configuration the dispatch uses: stages in flight per warp, CTAs per
// SM, queries in shared memory.
constexpr int ATT_STAGES = 2, ATT_MINB = 3;
constexpr bool ATT_QSMEM = true;

// Dynamic shared memory of one CTA: the scan arrays, then per warp its
// stages (raw code and meta rows for a quantised pool), the dequantised K or
// V tile (quantised pools) and the queries (qsmem).
size_t attn_smem(int nseq, int hd, int stages, bool qsmem, int bits, int row_bytes, int meta_row_bytes) {
  const size_t scan_bytes = ((size_t)2 * (nseq + 1) * 4 + 127) & ~(size_t)127;
  const size_t rowb = (size_t)hd * 2;
  const size_t stage = bits ? 2 * ATT_CHUNK * (size_t)(row_bytes + meta_row_bytes) : 2 * ATT_CHUNK * rowb;
  return scan_bytes + (size_t)ATT_WARPS * (stages * stage + (bits ? ATT_CHUNK * rowb : 0) +
                                           (qsmem ? ATT_CHUNK * rowb : 0));
}

// Quantised pools whose groups are too small to read as codes: the kernel
// that dequantises into a tile.
template <int DT, int HD>
AttnFn pick_attn(int bits, bool mf32) {
  if (bits == 8) return mf32 ? paged_decode_attn_kernel<DT, HD, ATT_STAGES, ATT_MINB, ATT_QSMEM, 8, true>
                             : paged_decode_attn_kernel<DT, HD, ATT_STAGES, ATT_MINB, ATT_QSMEM, 8, false>;
  return mf32 ? paged_decode_attn_kernel<DT, HD, ATT_STAGES, ATT_MINB, ATT_QSMEM, 4, true>
              : paged_decode_attn_kernel<DT, HD, ATT_STAGES, ATT_MINB, ATT_QSMEM, 4, false>;
}

AttnFn attn_kernel_of(const rmlx_pool_config& c) {
  const bool bf = c.dtype == RMLX_BF16, mf32 = c.meta_dtype == RMLX_F32;
  const int bits = c.quant_bits;
  return c.head_dim == 128 ? (bf ? pick_attn<RMLX_BF16, 128>(bits, mf32) : pick_attn<RMLX_F16, 128>(bits, mf32))
                           : (bf ? pick_attn<RMLX_BF16, 64>(bits, mf32) : pick_attn<RMLX_F16, 64>(bits, mf32));
}

// Quantised pools whose groups span whole k-steps and code columns are read
// as codes (paged_decode_attn_codes_kernel); the others are dequantised into
// a tile.
// CTAs per SM the register budget allows: two head tiles, or many groups,
// hold more accumulators
constexpr int cq_minb(int nh, int ng) { return nh == 2 ? 2 : (ng <= 2 ? 4 : 3); }
bool reads_codes(const rmlx_pool_config& c) {
  return (c.quant_bits == 8 && c.group_size >= 16) || (c.quant_bits == 4 && c.group_size >= 32);
}

constexpr int CQ_STAGES = 2;  // chunks in flight per warp
size_t attn_codes_smem(int nseq, int stages, int row_bytes, int meta_row_bytes) {
  const size_t scan_bytes = ((size_t)2 * (nseq + 1) * 4 + 127) & ~(size_t)127;
  const size_t stage = 2 * ATT_CHUNK * (size_t)(row_bytes + meta_row_bytes);
  return scan_bytes + (size_t)ATT_WARPS * stages * stage;
}

template <int HD, int BITS, int NH>
AttnFn pick_codes_gs(int gs) {
  if (gs == 16) {
    if constexpr (BITS == 8) return paged_decode_attn_codes_kernel<HD, 8, 16, NH, CQ_STAGES, cq_minb(NH, HD / 16)>;
    return nullptr;
  }
  if (gs == 32) return paged_decode_attn_codes_kernel<HD, BITS, 32, NH, CQ_STAGES, cq_minb(NH, HD / 32)>;
  if (gs == 64) return paged_decode_attn_codes_kernel<HD, BITS, 64, NH, CQ_STAGES, cq_minb(NH, HD / 64)>;
  if constexpr (HD == 128) {
    if (gs == 128) return paged_decode_attn_codes_kernel<HD, BITS, 128, NH, CQ_STAGES, cq_minb(NH, 1)>;
  }
  return nullptr;
}
template <int HD, int NH>
AttnFn pick_codes(const rmlx_pool_config& c) {
  return c.quant_bits == 8 ? pick_codes_gs<HD, 8, NH>(c.group_size) : pick_codes_gs<HD, 4, NH>(c.group_size);
}

// bf16/f16 pools: the transposed kernel, three CTAs of four warps per SM
// (two with two head tiles: more accumulators).
constexpr int RW_STAGES = 2;
template <int DT, int HD>
AttnFn pick_rows(int G) {
  return G <= 8 ? paged_decode_attn_rows_kernel<DT, HD, 1, RW_STAGES, 3>
                : paged_decode_attn_rows_kernel<DT, HD, 2, RW_STAGES, 2>;
}
size_t attn_rows_smem(int nseq, int hd) {
  const size_t scan_bytes = ((size_t)2 * (nseq + 1) * 4 + 127) & ~(size_t)127;
  return scan_bytes + (size_t)ATT_WARPS * RW_STAGES * 2 * ATT_CHUNK * hd * 2;
}

// The split kernel a pool's launches use and its dynamic shared memory.
struct AttnPlan {
  AttnFn fn;
  size_t smem;
  int items_x2;  // work items per resident warp, times 2 (attn_target)
};
AttnPlan attn_plan(const rmlx_kv_pool* p, int nseq, int G) {
  const rmlx_pool_config& c = p->cfg;
  const int hd = c.head_dim;
  if (reads_codes(c)) {
    AttnFn fn = hd == 128 ? (G <= 8 ? pick_codes<128, 1>(c) : pick_codes<128, 2>(c))
                          : (G <= 8 ? pick_codes<64, 1>(c) : pick_codes<64, 2>(c));
    if (fn)
      return {fn, attn_codes_smem(nseq, CQ_STAGES, (int)p->row_bytes, (int)p->meta_row_bytes),
              c.quant_bits == 8 ? 2 : 6};
  }
  if (!c.quant_bits) {
    const bool bf = c.dtype == RMLX_BF16;
    AttnFn fn = hd == 128 ? (bf ? pick_rows<RMLX_BF16, 128>(G) : pick_rows<RMLX_F16, 128>(G))
                          : (bf ? pick_rows<RMLX_BF16, 64>(G) : pick_rows<RMLX_F16, 64>(G));
    return {fn, attn_rows_smem(nseq, hd), 2};
  }
  return {attn_kernel_of(c),
          attn_smem(nseq, hd, ATT_STAGES, ATT_QSMEM, c.quant_bits, (int)p->row_bytes, (int)p->meta_row_bytes), 6};
}
}  // namespace

extern "C" {

rmlx_status rmlx_kv_attention_workspace_size(const rmlx_kv_pool* p, int32_t q_heads_per_kv, int32_t num_seqs,
                                             int64_t max_total_tokens, size_t* bytes) {
  if (!p || !bytes) return fail(RMLX_E_BAD_ARG, "NULL pool or bytes");
  if (q_heads_per_kv < 1 || q_heads_per_kv > 16) return fail(RMLX_E_BAD_ARG, "q_heads_per_kv must be in [1, 16]");
  if (num_seqs < 0 || max_total_tokens < 0) return fail(RMLX_E_BAD_ARG, "negative num_seqs or max_total_tokens");
  const rmlx_pool_config& c = p->cfg;
  int64_t splits = max_total_tokens / ATT_SPLIT + num_seqs;
  if ((c.dtype == RMLX_F16 || c.dtype == RMLX_BF16) && (c.head_dim == 64 || c.head_dim == 128)) {
    // room for the smaller splits a launch with few work items takes: the
    // last halving starts below the target, so at most twice it (4x kept)
    const AttnPlan plan = attn_plan(p, num_seqs, q_heads_per_kv);
    DeviceGuard dg(p->device);
    if (plan.smem <= 227 * 1024 && prepare_smem(plan.fn, plan.smem) == RMLX_OK) {
      const int64_t target = attn_target(plan.fn, plan.smem, p->num_sms, plan.items_x2);
      splits = std::max<int64_t>(splits, 4 * ((target + c.num_kv_heads - 1) / c.num_kv_heads) + num_seqs);
    }
  }
  *bytes = (size_t)splits * split_bytes(c.num_kv_heads, q_heads_per_kv, c.head_dim);
  return RMLX_OK;
}

rmlx_status rmlx_kv_decode_attention(rmlx_kv_pool* p, int32_t layer, const void* q, int32_t q_heads_per_kv,
                                     const int32_t* block_tables, int32_t block_table_stride, const int32_t* seq_lens,
                                     int32_t num_seqs, float softmax_scale, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  if (!p) return fail(RMLX_E_BAD_ARG, "NULL pool");
  const rmlx_pool_config& c = p->cfg;
  if (c.dtype != RMLX_F16 && c.dtype != RMLX_BF16) return fail(RMLX_E_BAD_ARG, "decode attention needs an F16 or BF16 pool");
  if (c.head_dim != 64 && c.head_dim != 128) return fail(RMLX_E_BAD_ARG, "decode attention supports head_dim 64 or 128");
  if (q_heads_per_kv < 1 || q_heads_per_kv > 16) return fail(RMLX_E_BAD_ARG, "q_heads_per_kv must be in [1, 16]");
  if (layer < 0 || layer >= c.num_layers) return fail(RMLX_E_RANGE, "layer %d out of range", layer);
  if (num_seqs < 0 || num_seqs > RMLX_MAX_SEQS_PER_LAUNCH) return fail(RMLX_E_BAD_ARG, "num_seqs out of range");
  if (num_seqs == 0) return RMLX_OK;
  if (!q || !out || !block_tables || !seq_lens || !workspace) return fail(RMLX_E_BAD_ARG, "NULL argument");
  if (!aligned16(q) || !aligned16(out) || !aligned16(workspace))
    return fail(RMLX_E_BAD_ARG, "q, out and workspace must be 16-byte aligned");
  if (block_table_stride < 0) return fail(RMLX_E_BAD_ARG, "negative block_table_stride");
  if (!(softmax_scale > 0.0f) || softmax_scale > 1e30f) return fail(RMLX_E_BAD_ARG, "softmax_scale must be positive");
  const int G = q_heads_per_kv, hd = c.head_dim, heads = c.num_kv_heads;
  const size_t per_split = split_bytes(heads, G, hd);
  const int64_t cap = (int64_t)(workspace_bytes / per_split);
  if (cap < 1) return fail(RMLX_E_BAD_ARG, "workspace smaller than one split");
  // partial outputs, then the (max, sum) pairs; heads x G x head_dim is a
  // multiple of 64 floats, so the second array starts 16-byte aligned
  float* part_o = static_cast<float*>(workspace);
  float* part_ml = part_o + (size_t)cap * heads * G * hd;
  DeviceGuard dg(p->device);
  cudaStream_t st = (cudaStream_t)stream;
  const bool bf = c.dtype == RMLX_BF16;
  const int bits = c.quant_bits;
  // one warp per (sequence, query head); with few pairs (each with many
  // splits: a launch over a shard of the KV heads) one CTA per pair, its
  // warps sharing the pair's splits.  Measured crossover: 512 pairs are
  // faster per CTA, 1024 per warp.
  const int64_t pairs = (int64_t)num_seqs * heads * G;
  const bool cta_combine = pairs < (int64_t)p->num_sms * 4;
  CombineFn fc = cta_combine
                     ? (hd == 128 ? (bf ? attn_combine_cta_kernel<RMLX_BF16, 128> : attn_combine_cta_kernel<RMLX_F16, 128>)
                                  : (bf ? attn_combine_cta_kernel<RMLX_BF16, 64> : attn_combine_cta_kernel<RMLX_F16, 64>))
                     : (hd == 128 ? (bf ? attn_combine_kernel<RMLX_BF16, 128> : attn_combine_kernel<RMLX_F16, 128>)
                                  : (bf ? attn_combine_kernel<RMLX_BF16, 64> : attn_combine_kernel<RMLX_F16, 64>));
  // p->attn_work, the item counter, is pool memory made by rmlx_kv_pool_new
  // and zero between launches: this call allocates nothing.
  rmlx_status s;
  if (p->attn_nseq != num_seqs || p->attn_G != G) {  // the launch shape, kept for the next call with the same shape
    const AttnPlan plan = attn_plan(p, num_seqs, G);
    if (plan.smem > 227 * 1024) return fail(RMLX_E_BAD_ARG, "num_seqs too large for one decode attention launch");
    if ((s = prepare_smem(plan.fn, plan.smem)) != RMLX_OK) return s;
    p->attn_fn = reinterpret_cast<void*>(plan.fn);
    p->attn_smem = plan.smem;
    p->attn_grid = persistent_grid(plan.fn, ATT_WARPS * 32, plan.smem, p->num_sms);
    p->attn_target = attn_target(plan.fn, plan.smem, p->num_sms, plan.items_x2);
    p->attn_nseq = num_seqs;
    p->attn_G = G;
  }
  AttnFn fa = reinterpret_cast<AttnFn>(p->attn_fn);
  const size_t smem = p->attn_smem;
  const int grid = p->attn_grid;
  const int64_t target = p->attn_target;
  const float scale_log2 = softmax_scale * 1.4426950408889634f;  // log2(e)
  cudaError_t e = launch_pdl(fa, dim3(grid), dim3(ATT_WARPS * 32), smem, st, p->geo(), (int)layer,
                             static_cast<const uint8_t*>(q), G, block_tables, (int)block_table_stride, seq_lens,
                             (int)num_seqs, target, scale_log2, part_o, part_ml, cap, static_cast<uint8_t*>(out),
                             bits ? log2i(c.group_size) : 0, p->attn_work, p->err);
  if (e != cudaSuccess) return cuda_check(e, "decode attention launch");
  const size_t csmem = cta_combine ? (size_t)((2 * (num_seqs + 1) + 3) & ~3) * 4 + (size_t)8 * (2 + hd) * 4
                                   : (size_t)2 * (num_seqs + 1) * 4;
  if ((s = prepare_smem(fc, csmem)) != RMLX_OK) return s;
  const int cgrid = cta_combine ? (int)pairs : (int)std::min<int64_t>((pairs + 7) / 8, (int64_t)p->num_sms * 8);
  e = launch_pdl(fc, dim3(cgrid), dim3(256), csmem, st, seq_lens, (int)num_seqs, target, heads, G, part_o,
                 part_ml, static_cast<uint8_t*>(out), cap, p->attn_work);
  if (e != cudaSuccess) {
    cudaMemsetAsync(p->attn_work, 0, 16, st);  // the combine would have reset the counter
    return cuda_check(e, "attention combine launch");
  }
  return cuda_check(cudaGetLastError(), "decode attention launch");
}

}  // extern "C"
