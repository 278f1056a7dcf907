// Paged KV pool on one B200: append (reshape-and-cache), block-table gather,
// fused group-affine quantise-on-append / dequantise-on-gather, block copy
// (copy-on-write / fork) and pack/unpack for migration.
//
// Reference semantics:
//   * append/gather move rows exactly like RotatingKVCache::append and
//     get_logical_order (crates/rmlx-serve-cache/src/rotating_cache.rs:
//     126-136, 162-197), with the row's position taken from a block table
//     instead of a ring buffer;
//   * the quantiser is quantize_group (quantized_cache.rs:232-273) applied
//     to each head_dim/group_size slice of a row: f32 min/max folds, scale =
//     range / (2^bits - 1) or 1.0 for a flat group, code = round-half-away(
//     (v - min) / scale) clamped, 4-bit codes packed low nibble first;
//   * the dequantiser is dequantize_group (:278-296): code * scale + zero as
//     a rounded multiply followed by a rounded add (no FMA), then rounded to
//     the output type.
//
// All kernels are HBM-bandwidth bound: 16-byte vector loads and stores,
// every warp streaming whole 4 KiB tiles, persistent grids sized from the
// SM count.  Tensor cores are not used (nothing here is a contraction).
#include <algorithm>
#include <new>

#include "dequant.cuh"
#include "kv_pool_internal.cuh"

namespace rmlx {


// ---------------------------------------------------------------------------
// Append: a CTA covers one layer (blockIdx.y) and a run of tokens; a (layer,
// token) pair is cpp = 2 x heads x (chunks per row) work units (K then V,
// head, chunk), which tile the CTA's threads (AppendShape): a thread takes
// unit x of token jt, jt + tpc, ... (APP tokens), loads all of them, then
// stores them.  Index arithmetic is 32-bit and done once per thread; the
// slot of each token is read once per thread.
// ---------------------------------------------------------------------------
constexpr int APPEND_APP = 4;  // tokens per thread

struct AppendShape {
  int cpp;    // work units per (layer, token)
  int tpc;    // tokens side by side in a CTA (cpp <= 256), else 1
  int iters;  // unit rounds per thread (cpp > 256: ceil(cpp / 256)), else 1
};

__device__ __forceinline__ void append_unit(const AppendShape& sh, int cpr, int heads, int it, int& x, int& jt,
                                            int& c, int& h, int& kv) {
  if (sh.tpc > 1) {
    jt = threadIdx.x / sh.cpp;
    x = threadIdx.x - jt * sh.cpp;
  } else {
    jt = 0;
    x = threadIdx.x + it * blockDim.x;
  }
  if (jt >= sh.tpc) x = sh.cpp;  // a thread past the last whole pair: no unit
  c = x % cpr;
  const int hk = x / cpr;
  h = hk % heads;
  kv = hk / heads;
}

__global__ void __launch_bounds__(256) append_rows_kernel(PoolGeo g, int l0, const uint8_t* __restrict__ k,
                                                          const uint8_t* __restrict__ v, int64_t ls, int64_t ts,
                                                          int64_t hs, const int32_t* __restrict__ slots, int T,
                                                          int cpr, AppendShape sh, int32_t* err) {
  pdl_wait();
  pdl_release();
  const int l = blockIdx.y;
  const int64_t cap = (int64_t)g.nblocks * g.bs;
  for (int it = 0; it < sh.iters; ++it) {
    int x, jt, c, h, kv;
    append_unit(sh, cpr, g.heads, it, x, jt, c, h, kv);
    const int t0 = blockIdx.x * sh.tpc * APPEND_APP + jt;
    int32_t s[APPEND_APP];
#pragma unroll
    for (int j = 0; j < APPEND_APP; ++j) {
      const int t = t0 + j * sh.tpc;
      s[j] = (x < sh.cpp && t < T) ? __ldg(slots + t) : -1;
      if (s[j] >= cap) {
        if (c == 0) atomicOr(err, DEV_ERR_SLOT);
        s[j] = -1;
      }
    }
    const uint8_t* src = (kv ? v : k) + l * ls + h * hs + c * 16;
    uint4 val[APPEND_APP];
#pragma unroll
    for (int j = 0; j < APPEND_APP; ++j)
      if (s[j] >= 0) val[j] = ld_stream(src + (int64_t)(t0 + j * sh.tpc) * ts);
#pragma unroll
    for (int j = 0; j < APPEND_APP; ++j) {
      if (s[j] < 0) continue;
      const int blk = s[j] / g.bs, off = s[j] - blk * g.bs;
      st_stream(g.base + g.tile_off(blk, l0 + l, kv, h) + (int64_t)off * g.row_bytes + c * 16, val[j]);
    }
  }
}


// ---------------------------------------------------------------------------
// Gather (plain): persistent CTAs, two CTAs of 256 threads per SM; each warp
// copies two (sequence block, kv, head) tiles per round with all 16 loads
// of a lane in flight before its stores.  Units are ordered with the head
// fastest so that a warp's two tiles (and its neighbours') are adjacent head
// tiles of one pool block; each full tile lands as one contiguous
// block_size * row_bytes run in the [seq][head][len][dim] output.
// ---------------------------------------------------------------------------
struct TileRef {
  const uint8_t* src;
  uint8_t* dst;
  int n16;
};

__device__ __forceinline__ TileRef gather_tile(const PoolGeo& g, int layer0, int nl, int64_t u, int64_t units,
                                               const int32_t* __restrict__ bt, int bt_stride, const int32_t* cub,
                                               const int32_t* cut, int nseq, uint8_t* ok, uint8_t* ov,
                                               int64_t out_row_bytes, int64_t out_layer_bytes, int lane,
                                               int32_t* err) {
  TileRef t{nullptr, nullptr, 0};
  if (u >= units) return t;
  // unit u = (layer l, gathered block gi, kv, head h), head fastest: a
  // layer's units follow the sequences' blocks as one layer's launch would
  // (measured 1 % faster than walking each block's layers in pool order)
  const int h = (int)(u % g.heads);
  int64_t q = u / g.heads;
  const int kv = (int)(q & 1);
  q >>= 1;
  int dl = 0;
  int64_t gi = q;
  if (nl > 1) {
    const int64_t nb = cub[nseq];
    dl = (int)(q / nb);
    gi = q - (int64_t)dl * nb;
  }
  const int s = find_seq(cub, nseq, gi);
  const int b = (int)(gi - cub[s]);
  const int L = cut[s + 1] - cut[s];
  const int32_t blk = __ldg(bt + (int64_t)s * bt_stride + b);
  if (blk < 0 || blk >= g.nblocks) {
    if (lane == 0) atomicOr(err, DEV_ERR_BLOCK);
    return t;
  }
  t.src = g.base + g.tile_off(blk, layer0 + dl, kv, h);
  t.dst = (kv ? ov : ok) + dl * out_layer_bytes +
          ((int64_t)cut[s] * g.heads + (int64_t)h * L + (int64_t)b * g.bs) * out_row_bytes;
  t.n16 = min(g.bs, L - b * g.bs) * g.row_bytes / 16;
  return t;
}

// nl layers from layer0 in one launch (rmlx_kv_gather: nl = 1); layer
// layer0 + i lands at out + i * out_layer_bytes.
__global__ void __launch_bounds__(256, 2) gather_rows_kernel(PoolGeo g, int layer0, int nl,
                                                             const int32_t* __restrict__ bt, int bt_stride,
                                                             const int32_t* __restrict__ lens, int nseq,
                                                             uint8_t* __restrict__ ok, uint8_t* __restrict__ ov,
                                                             int64_t out_layer_bytes, int32_t* err) {
  extern __shared__ int32_t smem[];
  int32_t* cub = smem;
  int32_t* cut = smem + nseq + 1;
  pdl_wait();
  pdl_release();
  scan_seq_lens(lens, nseq, g.bs, cub, cut);
  const int64_t units = (int64_t)cub[nseq] * nl * 2 * g.heads;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t u = ((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5) * 2; u < units; u += nwarps * 2) {
    const TileRef a = gather_tile(g, layer0, nl, u, units, bt, bt_stride, cub, cut, nseq, ok, ov, g.row_bytes,
                                  out_layer_bytes, lane, err);
    const TileRef b = gather_tile(g, layer0, nl, u + 1, units, bt, bt_stride, cub, cut, nseq, ok, ov, g.row_bytes,
                                  out_layer_bytes, lane, err);
    warp_copy2(a.src, a.dst, a.n16, b.src, b.dst, b.n16, lane);
  }
}

// ---------------------------------------------------------------------------
// Element conversions for the quantised paths.
// ---------------------------------------------------------------------------
template <int DT>  // rmlx_dtype
struct Elem;
template <>
struct Elem<RMLX_F32> {
  static constexpr int size = 4;
  // 8 consecutive elements -> f32
  __device__ __forceinline__ static void load8(const uint8_t* p, float* f) {
    uint4 a = ld_stream(p), b = ld_stream(p + 16);
    f[0] = __uint_as_float(a.x), f[1] = __uint_as_float(a.y), f[2] = __uint_as_float(a.z), f[3] = __uint_as_float(a.w);
    f[4] = __uint_as_float(b.x), f[5] = __uint_as_float(b.y), f[6] = __uint_as_float(b.z), f[7] = __uint_as_float(b.w);
  }
  __device__ __forceinline__ static void store8(uint8_t* p, const float* f) {
    st_stream(p, make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3])));
    st_stream(p + 16,
              make_uint4(__float_as_uint(f[4]), __float_as_uint(f[5]), __float_as_uint(f[6]), __float_as_uint(f[7])));
  }
};
template <>
struct Elem<RMLX_F16> {
  static constexpr int size = 2;
  __device__ __forceinline__ static void load8(const uint8_t* p, float* f) {
    uint4 a = ld_stream(p);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 x = __half22float2(h);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
  __device__ __forceinline__ static uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static void store8(uint8_t* p, const float* f) {
    st_stream(p, make_uint4(pack(f[0], f[1]), pack(f[2], f[3]), pack(f[4], f[5]), pack(f[6], f[7])));
  }
};
template <>
struct Elem<RMLX_BF16> {
  static constexpr int size = 2;
  __device__ __forceinline__ static void load8(const uint8_t* p, float* f) {
    uint4 a = ld_stream(p);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static void store8(uint8_t* p, const float* f) {
    st_stream(p, make_uint4(pack(f[0], f[1]), pack(f[2], f[3]), pack(f[4], f[5]), pack(f[6], f[7])));
  }
};

// Rust `x.round().clamp(0.0, qmax) as u8`: half-away rounding, clamp that
// passes NaN through, saturating cast with NaN -> 0.
__device__ __forceinline__ uint32_t quant_code(float v, float mn, float scale, float qmax) {
  float x = roundf(__fdiv_rn(__fsub_rn(v, mn), scale));
  if (x < 0.0f) x = 0.0f;
  if (x > qmax) x = qmax;
  return (x == x) ? (uint32_t)x : 0u;
}

// ---------------------------------------------------------------------------
// Quantise-on-append: one thread per 8 elements of a row, the CTAs laid out
// as for the plain append (one layer per blockIdx.y, AppendShape), one token
// per thread at a time; a group of group_size elements is group_size/8
// adjacent lanes (a power of two <= 32, aligned, never crossing a warp: the
// work units of a row are consecutive and a CTA's thread count is a multiple
// of 32), reduced with xor shuffles that every lane of the warp takes part
// in.
// ---------------------------------------------------------------------------
template <int IN_DT, int BITS, bool META_F32>
__global__ void __launch_bounds__(256) append_quant_kernel(PoolGeo g, int l0, const uint8_t* __restrict__ k,
                                                           const uint8_t* __restrict__ v, int64_t ls, int64_t ts,
                                                           int64_t hs, const int32_t* __restrict__ slots, int T,
                                                           int hd, int tpg, AppendShape sh, int32_t* err) {
  using E = Elem<IN_DT>;
  pdl_wait();
  pdl_release();
  const int cpr = hd / 8;
  const int l = blockIdx.y;
  const int64_t cap = (int64_t)g.nblocks * g.bs;
  const float qmax = (float)((1u << BITS) - 1);
  for (int it = 0; it < sh.iters; ++it) {
    int x, jt, c, h, kv;
    append_unit(sh, cpr, g.heads, it, x, jt, c, h, kv);
    const int t0 = blockIdx.x * sh.tpc * APPEND_APP + jt;
    const uint8_t* src = (kv ? v : k) + l * ls + h * hs + (int64_t)c * 8 * E::size;
    for (int j = 0; j < APPEND_APP; ++j) {
      const int t = t0 + j * sh.tpc;
      int32_t s = (x < sh.cpp && t < T) ? __ldg(slots + t) : -1;
      if (s >= cap) {
        if (c == 0) atomicOr(err, DEV_ERR_SLOT);
        s = -1;
      }
      const bool valid = s >= 0;
      float f[8];
      if (valid) {
        E::load8(src + (int64_t)t * ts, f);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = 0.0f;
      }
      float mx = -INFINITY, mn = INFINITY;
#pragma unroll
      for (int e = 0; e < 8; ++e) mx = fmaxf(mx, f[e]);
#pragma unroll
      for (int e = 0; e < 8; ++e) mn = fminf(mn, f[e]);
      for (int o = 1; o < tpg; o <<= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      }
      if (!valid) continue;
      const float range = __fsub_rn(mx, mn);
      const float scale = (range == 0.0f) ? 1.0f : __fdiv_rn(range, qmax);
      const int blk = s / g.bs, off = s - blk * g.bs;
      uint8_t* tile = g.base + g.tile_off(blk, l0 + l, kv, h);
      uint8_t* code_row = tile + (int64_t)off * g.row_bytes;
      if (BITS == 8) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) lo |= quant_code(f[e], mn, scale, qmax) << (8 * e);
#pragma unroll
        for (int e = 0; e < 4; ++e) hi |= quant_code(f[4 + e], mn, scale, qmax) << (8 * e);
        *reinterpret_cast<uint2*>(code_row + c * 8) = make_uint2(lo, hi);
      } else {
        uint32_t w = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t a = quant_code(f[2 * e], mn, scale, qmax), b = quant_code(f[2 * e + 1], mn, scale, qmax);
          w |= (a | (b << 4)) << (8 * e);
        }
        *reinterpret_cast<uint32_t*>(code_row + c * 4) = w;
      }
      if ((c & (tpg - 1)) == 0) {
        const int q = c / tpg;
        uint8_t* meta_row = tile + (int64_t)g.bs * g.row_bytes + (int64_t)off * g.meta_row_bytes;
        if (META_F32) {
          reinterpret_cast<float*>(meta_row)[2 * q] = scale;
          reinterpret_cast<float*>(meta_row)[2 * q + 1] = mn;
        } else {
          reinterpret_cast<__half2*>(meta_row)[q] = __halves2half2(__float2half_rn(scale), __float2half_rn(mn));
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Dequantise-on-gather.
//
// Per element the reference computes (code as f32) * scale + zero with a
// rounded multiply then a rounded add (dequantize_group).  The code's f32
// value comes from a byte permute that builds the bit pattern of 2^23 + code
// (exact for codes < 2^23) and an exact subtraction of 2^23, which keeps the
// slow conversion pipe out of the loop.  Then:
//  * f32 scale/zero: a rounded multiply and a rounded add (__fmul_rn,
//    __fadd_rn), exactly the reference's two steps;
//  * f16 scale/zero: code * scale is exact in f32 (a code has at most 8
//    significant bits and an f16 value 11, and the product stays inside
//    f32's normal range), so a fused multiply-add, which rounds once after
//    the add, gives the same result as the reference's multiply then add.
//    The kernel uses the packed forms (add.rn.f32x2, fma.rn.f32x2): one
//    instruction for two elements.
//
// Layout of the work: persistent CTAs, one warp per (sequence block, kv,
// head) tile.  A lane's task is one 16-byte segment of output (8 bf16/f16
// or 4 f32 elements) and the code bytes behind it, so consecutive lanes
// write consecutive 16 bytes (every store instruction covers 512 contiguous
// bytes) and read consecutive code bytes.  group_size >= 8 and a power of
// two, so a task never straddles a (scale, zero) group.  All of a round's
// loads (codes and scale/zero) are issued before its first store.
//
// Task indexing (IDX): with tpr tasks per row, a task's row and group are
// found by division (0: tpr not a power of two), by shifts (1), or, when
// tpr divides 32 (2: the common head_dim 128 with 16-bit output), from
// per-lane constants: a lane's group is the same in every round step and
// its row advances by 32 / tpr rows per step.
// ---------------------------------------------------------------------------

template <bool META_F32>
__device__ __forceinline__ void meta_at(const uint8_t* mrow, int gq, float& sc, float& zr) {
  if (META_F32) {
    const float2 m = __ldg(reinterpret_cast<const float2*>(mrow) + gq);
    sc = m.x;
    zr = m.y;
  } else {
    const float2 m = __half22float2(__ldg(reinterpret_cast<const __half2*>(mrow) + gq));
    sc = m.x;
    zr = m.y;
  }
}

// Non-coherent loads of the code bytes of one task (2, 4 or 8 bytes).
template <int CB>
__device__ __forceinline__ uint2 load_codes(const uint8_t* p) {
  uint2 r = make_uint2(0u, 0u);
  if (CB == 8) {
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  } else if (CB == 4) {
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r.x) : "l"(p));
  } else {
    unsigned short h;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(h) : "l"(p));
    r.x = h;
  }
  return r;
}

template <int DT>
struct Store16;  // 16 bytes of output from f32 values, round-to-nearest-even
template <>
struct Store16<RMLX_F32> {
  static constexpr int n = 4;
  __device__ __forceinline__ static void run(uint8_t* p, const float* f) {
    st_stream(p, make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                            __float_as_uint(f[3])));
  }
};
template <>
struct Store16<RMLX_F16> {
  static constexpr int n = 8;
  __device__ __forceinline__ static void run(uint8_t* p, const float* f) { Elem<RMLX_F16>::store8(p, f); }
};
template <>
struct Store16<RMLX_BF16> {
  static constexpr int n = 8;
  __device__ __forceinline__ static void run(uint8_t* p, const float* f) { Elem<RMLX_BF16>::store8(p, f); }
};

// One round of a warp over TPW tiles: tasks base + lane + 32 v (v < V) of
// each tile.  All loads (codes, scale/zero) are issued before the first store.
// Task t reads code bytes [t * CB, (t + 1) * CB) (code rows are contiguous)
// and writes output bytes [16 t, 16 t + 16) (the tile's output rows are
// contiguous too).  base is a multiple of 32 * V.
template <int BITS, int OUT_DT, bool META_F32, int IDX, int TPW, int V>
__device__ __forceinline__ void dq_round(const PoolGeo& g, const uint8_t* const* tile, uint8_t* const* out,
                                         const int* ntasks, int base, int lane, int tpr, int tpr_log2, int gs_log2) {
  constexpr int EPT = Store16<OUT_DT>::n;  // output elements per task (16 bytes)
  constexpr int CB = EPT * BITS / 8;       // code bytes per task
  constexpr int MSZ = META_F32 ? 8 : 4;    // bytes of one (scale, zero) pair
  const int meta_off = g.bs * g.row_bytes;
  const int mrb = g.meta_row_bytes;
  const int t0 = base + lane;
  // IDX 2: byte offset of this lane's (scale, zero) in the tile at v = 0,
  // and its advance per v.
  int moff = 0, mstep = 0;
  if (IDX == 2) {
    moff = meta_off + (t0 >> tpr_log2) * mrb + (((lane & (tpr - 1)) * EPT) >> gs_log2) * MSZ;
    mstep = (32 >> tpr_log2) * mrb;
  }
  uint2 cw[TPW][V];
  float sc[TPW][V], zr[TPW][V];
#pragma unroll
  for (int k = 0; k < TPW; ++k) {
    const uint8_t* cbase = tile[k] + t0 * CB;
    const uint8_t* mbase = tile[k] + moff;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int t = t0 + 32 * v;
      cw[k][v] = make_uint2(0u, 0u);
      sc[k][v] = zr[k][v] = 0.0f;
      if (t < ntasks[k]) {
        cw[k][v] = load_codes<CB>(cbase + 32 * CB * v);
        if (IDX == 2) {
          meta_at<META_F32>(mbase + v * mstep, 0, sc[k][v], zr[k][v]);
        } else {
          const int r = IDX ? (t >> tpr_log2) : t / tpr;
          const int e0 = (IDX ? (t & (tpr - 1)) : (t - r * tpr)) * EPT;
          meta_at<META_F32>(tile[k] + meta_off + r * mrb, e0 >> gs_log2, sc[k][v], zr[k][v]);
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < TPW; ++k) {
    uint8_t* obase = out[k] + (int64_t)t0 * 16;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (t0 + 32 * v >= ntasks[k]) continue;
      uint32_t lo4 = 0, hi4 = 0;
      if (BITS == 4) {
        lo4 = cw[k][v].x & 0x0F0F0F0Fu;
        hi4 = (cw[k][v].x >> 4) & 0x0F0F0F0Fu;
      }
      if (OUT_DT == RMLX_F32) {
        float f[4];
        dq_pair<BITS, META_F32>(cw[k][v], lo4, hi4, 0, sc[k][v], zr[k][v], f[0], f[1]);
        dq_pair<BITS, META_F32>(cw[k][v], lo4, hi4, 2, sc[k][v], zr[k][v], f[2], f[3]);
        Store16<RMLX_F32>::run(obase + 512 * v, f);
      } else {  // 16-bit output: each pair packed as soon as it is computed
        uint32_t w[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          float a, b;
          dq_pair<BITS, META_F32>(cw[k][v], lo4, hi4, 2 * p, sc[k][v], zr[k][v], a, b);
          w[p] = Elem<OUT_DT == RMLX_F32 ? RMLX_BF16 : OUT_DT>::pack(a, b);
        }
        st_stream(obase + 512 * v, make_uint4(w[0], w[1], w[2], w[3]));
      }
    }
  }
}

// The common case as its own kernel: every tile fits one round (block_size *
// tasks per row <= 32 * V) and tasks per row divide 32, so a lane's code,
// (scale, zero) and output addresses are per-lane constants plus immediate
// offsets.  Same tasks, loads and arithmetic as gather_dequant_kernel.
template <int BITS, int OUT_DT, bool META_F32>
__global__ void __launch_bounds__(256, 2) gather_dequant_r1_kernel(PoolGeo g, int layer, const int32_t* __restrict__ bt,
                                                                   int bt_stride, const int32_t* __restrict__ lens,
                                                                   int nseq, uint8_t* __restrict__ ok,
                                                                   uint8_t* __restrict__ ov, int hd, int gs_log2,
                                                                   int tpr_log2, int32_t* err) {
  constexpr int EPT = Store16<OUT_DT>::n;
  constexpr int CB = EPT * BITS / 8;
  constexpr int MSZ = META_F32 ? 8 : 4;
  constexpr int V = 8, TPW = 2;
  extern __shared__ int32_t smem[];
  int32_t* cub = smem;
  int32_t* cut = smem + nseq + 1;
  pdl_wait();
  pdl_release();
  scan_seq_lens(lens, nseq, g.bs, cub, cut);
  const int64_t units = (int64_t)cub[nseq] * 2 * g.heads;
  const bool units32 = units <= (int64_t)UINT32_MAX;
  const int lane = threadIdx.x & 31;
  const int tpr = 1 << tpr_log2;
  const int mrb = g.meta_row_bytes;
  const int64_t orb = (int64_t)hd * (16 / EPT);
  // per-lane constants: code offset, (scale, zero) offset and its advance per v
  const int coff = lane * CB;
  const int moff = g.bs * g.row_bytes + (lane >> tpr_log2) * mrb + (((lane & (tpr - 1)) * EPT) >> gs_log2) * MSZ;
  const int mstep = (32 >> tpr_log2) * mrb;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t u0 = ((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5) * TPW; u0 < units;
       u0 += nwarps * TPW) {
    const uint8_t* tile[TPW];
    uint8_t* out[TPW];
    int ntasks[TPW];
#pragma unroll
    for (int k = 0; k < TPW; ++k) {
      const int64_t u = u0 + k;
      tile[k] = g.base;
      out[k] = ok;
      ntasks[k] = 0;
      if (u >= units) continue;
      int h, kv;
      int64_t gi;
      if (units32) {
        const uint32_t uu = (uint32_t)u, hh = (uint32_t)g.heads, q = uu / hh;
        h = (int)(uu - q * hh);
        kv = (int)(q & 1u);
        gi = (int64_t)(q >> 1);
      } else {
        h = (int)(u % g.heads);
        const int64_t q = u / g.heads;
        kv = (int)(q & 1);
        gi = q >> 1;
      }
      const int s = find_seq(cub, nseq, gi);
      const int b = (int)(gi - cub[s]);
      const int L = cut[s + 1] - cut[s];
      const int32_t blk = __ldg(bt + (int64_t)s * bt_stride + b);
      if (blk < 0 || blk >= g.nblocks) {
        if (lane == 0) atomicOr(err, DEV_ERR_BLOCK);
        continue;
      }
      tile[k] = g.base + g.tile_off(blk, layer, kv, h);
      out[k] = (kv ? ov : ok) + ((int64_t)cut[s] * g.heads + (int64_t)h * L + (int64_t)b * g.bs) * orb;
      ntasks[k] = min(g.bs, L - b * g.bs) << tpr_log2;
    }
    uint2 cw[TPW][V];
    float sc[TPW][V], zr[TPW][V];
#pragma unroll
    for (int k = 0; k < TPW; ++k) {
      const uint8_t* cbase = tile[k] + coff;
      const uint8_t* mbase = tile[k] + moff;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        cw[k][v] = make_uint2(0u, 0u);
        sc[k][v] = zr[k][v] = 0.0f;
        if (lane + 32 * v < ntasks[k]) {
          cw[k][v] = load_codes<CB>(cbase + 32 * CB * v);
          meta_at<META_F32>(mbase + v * mstep, 0, sc[k][v], zr[k][v]);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < TPW; ++k) {
      uint8_t* obase = out[k] + lane * 16;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        if (lane + 32 * v >= ntasks[k]) continue;
        uint32_t lo4 = 0, hi4 = 0;
        if (BITS == 4) {
          lo4 = cw[k][v].x & 0x0F0F0F0Fu;
          hi4 = (cw[k][v].x >> 4) & 0x0F0F0F0Fu;
        }
        if (OUT_DT == RMLX_F32) {
          float f[4];
          dq_pair<BITS, META_F32>(cw[k][v], lo4, hi4, 0, sc[k][v], zr[k][v], f[0], f[1]);
          dq_pair<BITS, META_F32>(cw[k][v], lo4, hi4, 2, sc[k][v], zr[k][v], f[2], f[3]);
          Store16<RMLX_F32>::run(obase + 512 * v, f);
        } else {
          uint32_t w[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            float a, b;
            dq_pair<BITS, META_F32>(cw[k][v], lo4, hi4, 2 * p, sc[k][v], zr[k][v], a, b);
            w[p] = Elem<OUT_DT == RMLX_F32 ? RMLX_BF16 : OUT_DT>::pack(a, b);
          }
          st_stream(obase + 512 * v, make_uint4(w[0], w[1], w[2], w[3]));
        }
      }
    }
  }
}

template <int BITS, int OUT_DT, bool META_F32, int IDX>
__global__ void __launch_bounds__(256, 2) gather_dequant_kernel(PoolGeo g, int layer, const int32_t* __restrict__ bt,
                                                                int bt_stride, const int32_t* __restrict__ lens,
                                                                int nseq, uint8_t* __restrict__ ok,
                                                                uint8_t* __restrict__ ov, int hd, int gs_log2,
                                                                int tpr_log2, int32_t* err) {
  constexpr int EPT = Store16<OUT_DT>::n;
  constexpr int V = 8;    // tasks per lane per tile per round
  constexpr int TPW = 2;  // tiles per warp per round
  extern __shared__ int32_t smem[];
  int32_t* cub = smem;
  int32_t* cut = smem + nseq + 1;
  pdl_wait();
  pdl_release();
  scan_seq_lens(lens, nseq, g.bs, cub, cut);
  const int64_t units = (int64_t)cub[nseq] * 2 * g.heads;
  const bool units32 = units <= (int64_t)UINT32_MAX;  // uniform: 32-bit unit arithmetic
  const int lane = threadIdx.x & 31;
  const int tpr = hd / EPT;  // tasks per row
  const int64_t orb = (int64_t)hd * (16 / EPT);
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t u0 = ((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5) * TPW; u0 < units;
       u0 += nwarps * TPW) {
    const uint8_t* tile[TPW];
    uint8_t* out[TPW];
    int ntasks[TPW];
    int nmax = 0;
#pragma unroll
    for (int k = 0; k < TPW; ++k) {
      const int64_t u = u0 + k;
      tile[k] = nullptr;
      out[k] = nullptr;
      ntasks[k] = 0;
      if (u >= units) continue;
      // unit u = (gathered block gi, kv, head h), head fastest
      int h, kv;
      int64_t gi;
      if (units32) {
        const uint32_t uu = (uint32_t)u, hh = (uint32_t)g.heads, q = uu / hh;
        h = (int)(uu - q * hh);
        kv = (int)(q & 1u);
        gi = (int64_t)(q >> 1);
      } else {
        h = (int)(u % g.heads);
        const int64_t q = u / g.heads;
        kv = (int)(q & 1);
        gi = q >> 1;
      }
      const int s = find_seq(cub, nseq, gi);
      const int b = (int)(gi - cub[s]);
      const int L = cut[s + 1] - cut[s];
      const int32_t blk = __ldg(bt + (int64_t)s * bt_stride + b);
      if (blk < 0 || blk >= g.nblocks) {
        if (lane == 0) atomicOr(err, DEV_ERR_BLOCK);
        continue;
      }
      tile[k] = g.base + g.tile_off(blk, layer, kv, h);
      out[k] = (kv ? ov : ok) + ((int64_t)cut[s] * g.heads + (int64_t)h * L + (int64_t)b * g.bs) * orb;
      ntasks[k] = min(g.bs, L - b * g.bs) * tpr;
      nmax = max(nmax, ntasks[k]);
    }
    if (nmax <= 32 * V) {
      dq_round<BITS, OUT_DT, META_F32, IDX, TPW, V>(g, tile, out, ntasks, 0, lane, tpr, tpr_log2, gs_log2);
    } else {
      for (int base = 0; base < nmax; base += 32 * V)
        dq_round<BITS, OUT_DT, META_F32, IDX, TPW, V>(g, tile, out, ntasks, base, lane, tpr, tpr_log2, gs_log2);
    }
  }
}

// ---------------------------------------------------------------------------
// Block copy / pack / unpack: a warp copies two 4 KiB segments per round.
//   mode 0: pool[dst[i]] = pool[src[i]]
//   mode 1: staging[i]   = pool[src[i]]       (pack)
//   mode 2: pool[src[i]] = staging[i]         (unpack)
// ---------------------------------------------------------------------------
__device__ __forceinline__ TileRef copy_segment(uint8_t* base, int64_t block_bytes, int nblocks,
                                                const int32_t* __restrict__ src, const int32_t* __restrict__ dst,
                                                int64_t u, int64_t units, int64_t segs, int mode, uint8_t* staging,
                                                int lane, int32_t* err) {
  TileRef t{nullptr, nullptr, 0};
  if (u >= units) return t;
  const int i = (int)(u / segs);
  const int64_t off = (u - (int64_t)i * segs) * 4096;
  const int32_t a = __ldg(src + i);
  const int32_t b = mode == 0 ? __ldg(dst + i) : 0;
  if (a < 0 || a >= nblocks || b < 0 || b >= nblocks) {
    if (lane == 0 && off == 0) atomicOr(err, DEV_ERR_BLOCK);
    return t;
  }
  if (mode == 0) {
    t.src = base + (int64_t)a * block_bytes + off;
    t.dst = base + (int64_t)b * block_bytes + off;
  } else if (mode == 1) {
    t.src = base + (int64_t)a * block_bytes + off;
    t.dst = staging + (int64_t)i * block_bytes + off;
  } else {
    t.src = staging + (int64_t)i * block_bytes + off;
    t.dst = base + (int64_t)a * block_bytes + off;
  }
  t.n16 = (int)(min((int64_t)4096, block_bytes - off) / 16);
  return t;
}

__global__ void __launch_bounds__(256, 2) copy_blocks_kernel(uint8_t* base, int64_t block_bytes, int nblocks,
                                                             const int32_t* __restrict__ src,
                                                             const int32_t* __restrict__ dst, int n, int mode,
                                                             uint8_t* staging, int32_t* err) {
  pdl_wait();
  pdl_release();
  const int64_t segs = (block_bytes + 4095) / 4096;
  const int64_t units = (int64_t)n * segs;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t u = ((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5) * 2; u < units; u += nwarps * 2) {
    const TileRef a = copy_segment(base, block_bytes, nblocks, src, dst, u, units, segs, mode, staging, lane, err);
    const TileRef b = copy_segment(base, block_bytes, nblocks, src, dst, u + 1, units, segs, mode, staging, lane, err);
    warp_copy2(a.src, a.dst, a.n16, b.src, b.dst, b.n16, lane);
  }
}

static int dtype_size(int dt) { return dt == RMLX_F32 ? 4 : 2; }

}  // namespace rmlx

using namespace rmlx;


namespace {

// Dispatch tables for the templated quantised kernels.
using AppendQuantFn = void (*)(PoolGeo, int, const uint8_t*, const uint8_t*, int64_t, int64_t, int64_t,
                               const int32_t*, int, int, int, AppendShape, int32_t*);
template <int IN, int BITS, bool MF32>
AppendQuantFn aq() {
  return append_quant_kernel<IN, BITS, MF32>;
}
AppendQuantFn pick_append_quant(int in_dt, int bits, bool mf32) {
  static const AppendQuantFn t[3][2][2] = {
      {{aq<0, 4, false>(), aq<0, 4, true>()}, {aq<0, 8, false>(), aq<0, 8, true>()}},
      {{aq<1, 4, false>(), aq<1, 4, true>()}, {aq<1, 8, false>(), aq<1, 8, true>()}},
      {{aq<2, 4, false>(), aq<2, 4, true>()}, {aq<2, 8, false>(), aq<2, 8, true>()}},
  };
  return t[in_dt][bits == 8][mf32];
}

using GatherDqFn = void (*)(PoolGeo, int, const int32_t*, int, const int32_t*, int, uint8_t*, uint8_t*, int, int,
                            int, int32_t*);
template <int BITS, int OUT, bool MF32, int IDX>
GatherDqFn gd() {
  return gather_dequant_kernel<BITS, OUT, MF32, IDX>;
}
template <int BITS, int OUT, bool MF32>
GatherDqFn gd1() {
  return gather_dequant_r1_kernel<BITS, OUT, MF32>;
}
GatherDqFn pick_gather_dequant_r1(int bits, int out_dt, bool mf32) {
#define GD1_ROW(B, O) {gd1<B, O, false>(), gd1<B, O, true>()}
  static const GatherDqFn t[2][3][2] = {
      {GD1_ROW(4, 0), GD1_ROW(4, 1), GD1_ROW(4, 2)},
      {GD1_ROW(8, 0), GD1_ROW(8, 1), GD1_ROW(8, 2)},
  };
#undef GD1_ROW
  return t[bits == 8][out_dt][mf32];
}
// idx: 0 = tpr not a power of two, 1 = power of two above 32, 2 = divides 32
GatherDqFn pick_gather_dequant(int bits, int out_dt, bool mf32, int idx) {
#define GD_M(B, O, M) {gd<B, O, M, 0>(), gd<B, O, M, 1>(), gd<B, O, M, 2>()}
#define GD_ROW(B, O) {GD_M(B, O, false), GD_M(B, O, true)}
  static const GatherDqFn t[2][3][2][3] = {
      {GD_ROW(4, 0), GD_ROW(4, 1), GD_ROW(4, 2)},
      {GD_ROW(8, 0), GD_ROW(8, 1), GD_ROW(8, 2)},
  };
#undef GD_ROW
#undef GD_M
  return t[bits == 8][out_dt][mf32][idx];
}

}  // namespace

extern "C" {

rmlx_status rmlx_kv_pool_new(const rmlx_pool_config* cfg, int device, rmlx_kv_pool** out) {
  if (!cfg || !out) return fail(RMLX_E_BAD_ARG, "NULL cfg or out");
  *out = nullptr;
  const rmlx_pool_config c = *cfg;
  if (c.num_layers <= 0 || c.num_kv_heads <= 0 || c.head_dim <= 0 || c.block_size <= 0 || c.num_blocks <= 0)
    return fail(RMLX_E_BAD_ARG, "pool dimensions must be positive");
  if (c.dtype < RMLX_F32 || c.dtype > RMLX_BF16) return fail(RMLX_E_BAD_ARG, "dtype must be F32, F16 or BF16");
  if ((int64_t)c.num_blocks * c.block_size > INT32_MAX) return fail(RMLX_E_BAD_ARG, "num_blocks * block_size exceeds int32 slots");
  rmlx_kv_pool p;
  p.cfg = c;
  p.device = device;
  if (c.quant_bits == 0) {
    p.row_bytes = (size_t)c.head_dim * dtype_size(c.dtype);
    if (p.row_bytes % 16) return fail(RMLX_E_BAD_ARG, "head_dim * element size must be a multiple of 16 bytes");
    p.meta_row_bytes = 0;
  } else if (c.quant_bits == 4 || c.quant_bits == 8) {
    if (!is_pow2(c.group_size) || c.group_size < 8 || c.group_size > 256)
      return fail(RMLX_E_BAD_ARG, "group_size must be a power of two in [8, 256]");
    if (c.head_dim % c.group_size) return fail(RMLX_E_BAD_ARG, "head_dim must be a multiple of group_size");
    if (c.meta_dtype != RMLX_F32 && c.meta_dtype != RMLX_F16) return fail(RMLX_E_BAD_ARG, "meta_dtype must be F32 or F16");
    p.row_bytes = (size_t)c.head_dim * c.quant_bits / 8;
    if (p.row_bytes % 16) return fail(RMLX_E_BAD_ARG, "head_dim * bits / 8 must be a multiple of 16 bytes");
    p.meta_row_bytes = (size_t)(c.head_dim / c.group_size) * 2 * dtype_size(c.meta_dtype);
  } else {
    return fail(RMLX_E_BAD_ARG, "bits must be 4 or 8, got %d", c.quant_bits);
  }
  p.tile_bytes = ((size_t)c.block_size * (p.row_bytes + p.meta_row_bytes) + 15) / 16 * 16;
  p.block_bytes = p.tile_bytes * c.num_layers * 2 * c.num_kv_heads;
  p.bytes = p.block_bytes * c.num_blocks;
  DeviceGuard dg(device);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0) p.num_sms = sms;
  rmlx_status s = cuda_check(cudaMalloc(&p.base, p.bytes), "cudaMalloc(pool)");
  if (s != RMLX_OK) return s == RMLX_E_CUDA ? fail(RMLX_E_EXHAUSTED, "%s", rmlx_last_error()) : s;
  if ((s = cuda_check(cudaMalloc(&p.err, sizeof(int32_t)), "cudaMalloc(err)")) != RMLX_OK) {
    cudaFree(p.base);
    return s;
  }
  // The decode attention's work-item counter lives with the pool, so that no
  // attention call allocates (a first call may then sit inside a stream
  // capture); the kernels leave it at zero between launches.
  void* work = nullptr;
  if ((s = cuda_check(cudaMalloc(&work, 16), "cudaMalloc(attention counter)")) != RMLX_OK) {
    cudaFree(p.base);
    cudaFree(p.err);
    return s;
  }
  p.attn_work = static_cast<unsigned long long*>(work);
  if ((s = cuda_check(cudaMemset(p.base, 0, p.bytes), "cudaMemset(pool)")) != RMLX_OK ||
      (s = cuda_check(cudaMemset(p.err, 0, sizeof(int32_t)), "cudaMemset(err)")) != RMLX_OK ||
      (s = cuda_check(cudaMemset(p.attn_work, 0, 16), "cudaMemset(attention counter)")) != RMLX_OK) {
    cudaFree(p.base);
    cudaFree(p.err);
    cudaFree(p.attn_work);
    return s;
  }
  *out = new (std::nothrow) rmlx_kv_pool(p);
  if (!*out) {
    cudaFree(p.base);
    cudaFree(p.err);
    cudaFree(p.attn_work);
    return fail(RMLX_E_EXHAUSTED, "host allocation failed");
  }
  return RMLX_OK;
}

void rmlx_kv_pool_destroy(rmlx_kv_pool* p) {
  if (!p) return;
  {
    DeviceGuard dg(p->device);
    cudaFree(p->base);
    cudaFree(p->err);
    cudaFree(p->attn_work);
  }
  delete p;
}

rmlx_status rmlx_kv_pool_layout(const rmlx_kv_pool* p, rmlx_pool_layout* o) {
  if (!p || !o) return fail(RMLX_E_BAD_ARG, "NULL pool or out");
  o->base = p->base;
  o->bytes = p->bytes;
  o->tile_bytes = p->tile_bytes;
  o->block_bytes = p->block_bytes;
  o->row_bytes = p->row_bytes;
  o->meta_row_bytes = p->meta_row_bytes;
  return RMLX_OK;
}

rmlx_status rmlx_kv_pool_check(rmlx_kv_pool* p, int32_t* device_error) {
  if (!p || !device_error) return fail(RMLX_E_BAD_ARG, "NULL pool or out");
  DeviceGuard dg(p->device);
  rmlx_status s = cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  if (s != RMLX_OK) return s;
  if ((s = cuda_check(cudaMemcpy(device_error, p->err, sizeof(int32_t), cudaMemcpyDeviceToHost), "read error word")) != RMLX_OK)
    return s;
  return cuda_check(cudaMemset(p->err, 0, sizeof(int32_t)), "clear error word");
}

rmlx_status rmlx_kv_pool_status_async(rmlx_kv_pool* p, int32_t* status, void* stream) {
  if (!p || !status) return fail(RMLX_E_BAD_ARG, "NULL pool or status");
  DeviceGuard dg(p->device);
  return cuda_check(
      cudaMemcpyAsync(status, p->err, sizeof(int32_t), cudaMemcpyDeviceToHost, (cudaStream_t)stream),
      "read error word");
}

rmlx_status rmlx_kv_pool_read(rmlx_kv_pool* p, size_t offset, size_t nbytes, void* host_dst) {
  if (!p || (nbytes && !host_dst)) return fail(RMLX_E_BAD_ARG, "NULL pool or destination");
  if (offset > p->bytes || nbytes > p->bytes - offset) return fail(RMLX_E_RANGE, "read past the end of the pool");
  if (nbytes == 0) return RMLX_OK;
  DeviceGuard dg(p->device);
  return cuda_check(cudaMemcpy(host_dst, p->base + offset, nbytes, cudaMemcpyDeviceToHost), "pool read");
}

rmlx_status rmlx_kv_pool_write(rmlx_kv_pool* p, size_t offset, size_t nbytes, const void* host_src) {
  if (!p || (nbytes && !host_src)) return fail(RMLX_E_BAD_ARG, "NULL pool or source");
  if (offset > p->bytes || nbytes > p->bytes - offset) return fail(RMLX_E_RANGE, "write past the end of the pool");
  if (nbytes == 0) return RMLX_OK;
  DeviceGuard dg(p->device);
  return cuda_check(cudaMemcpy(p->base + offset, host_src, nbytes, cudaMemcpyHostToDevice), "pool write");
}

rmlx_status rmlx_kv_append(rmlx_kv_pool* p, int32_t layer_begin, int32_t num_layers, const void* k, const void* v,
                           int64_t layer_stride, int64_t token_stride, int64_t head_stride, const int32_t* slots,
                           int32_t T, void* stream) {
  if (!p) return fail(RMLX_E_BAD_ARG, "NULL pool");
  const rmlx_pool_config& c = p->cfg;
  if (layer_begin < 0 || num_layers < 0 || layer_begin + num_layers > c.num_layers)
    return fail(RMLX_E_RANGE, "layers [%d, %d) outside the pool's %d layers", layer_begin, layer_begin + num_layers,
                c.num_layers);
  if (T < 0) return fail(RMLX_E_BAD_ARG, "num_tokens < 0");
  if (T == 0 || num_layers == 0) return RMLX_OK;
  if (!k || !v || !slots) return fail(RMLX_E_BAD_ARG, "NULL k, v or slot_mapping");
  const int es = dtype_size(c.dtype);
  const int64_t ls = layer_stride * es, ts = token_stride * es, hs = head_stride * es;
  if (!aligned16(k) || !aligned16(v) || (ls % 16) || (ts % 16) || (hs % 16))
    return fail(RMLX_E_BAD_ARG, "k/v pointers and strides must be 16-byte aligned");
  DeviceGuard dg(p->device);
  cudaStream_t st = (cudaStream_t)stream;
  PoolGeo g = p->geo();
  const uint8_t* kb = (const uint8_t*)k;
  const uint8_t* vb = (const uint8_t*)v;
  if (num_layers > 65535) return fail(RMLX_E_BAD_ARG, "more than 65535 layers in one append");
  // work units per (layer, token): 16-byte chunks (plain) or 8-element
  // chunks (quantised) of the K and V rows of every head
  const int cpr = c.quant_bits == 0 ? (int)(p->row_bytes / 16) : c.head_dim / 8;
  AppendShape sh;
  sh.cpp = 2 * c.num_kv_heads * cpr;
  int block;
  if (sh.cpp <= 256) {
    sh.tpc = 256 / sh.cpp;
    sh.iters = 1;
    block = (sh.tpc * sh.cpp + 31) / 32 * 32;
  } else {
    sh.tpc = 1;
    sh.iters = (sh.cpp + 255) / 256;
    block = 256;
  }
  const dim3 grid((unsigned)((T + sh.tpc * APPEND_APP - 1) / (sh.tpc * APPEND_APP)), (unsigned)num_layers);
  if (c.quant_bits == 0) {
    cudaError_t e = launch_pdl(append_rows_kernel, grid, dim3(block), 0, st, g, layer_begin, kb, vb, ls, ts, hs, slots,
                               T, cpr, sh, p->err);
    if (e != cudaSuccess) return cuda_check(e, "append launch");
  } else {
    const int tpg = c.group_size / 8;
    AppendQuantFn fn = pick_append_quant(c.dtype, c.quant_bits, c.meta_dtype == RMLX_F32);
    cudaError_t e = launch_pdl(fn, grid, dim3(block), 0, st, g, layer_begin, kb, vb, ls, ts, hs, slots, T,
                               c.head_dim, tpg, sh, p->err);
    if (e != cudaSuccess) return cuda_check(e, "append launch");
  }
  return cuda_check(cudaGetLastError(), "append launch");
}

static rmlx_status gather_impl(rmlx_kv_pool* p, int32_t layer, int32_t nl, const int32_t* bt, int32_t bt_stride,
                               const int32_t* lens, int32_t nseq, void* out_k, void* out_v, int64_t out_layer_stride,
                               void* stream) {
  if (!p) return fail(RMLX_E_BAD_ARG, "NULL pool");
  const rmlx_pool_config& c = p->cfg;
  if (layer < 0 || nl < 0 || layer + nl > c.num_layers)
    return fail(RMLX_E_RANGE, "layers [%d, %d) outside the pool's %d layers", layer, layer + nl, c.num_layers);
  if (nseq < 0 || nseq > RMLX_MAX_SEQS_PER_LAUNCH)
    return fail(RMLX_E_BAD_ARG, "num_seqs %d outside [0, %d]", nseq, RMLX_MAX_SEQS_PER_LAUNCH);
  if (nseq == 0 || nl == 0) return RMLX_OK;
  if (!bt || !lens || !out_k || !out_v) return fail(RMLX_E_BAD_ARG, "NULL block_tables, seq_lens or outputs");
  if (bt_stride < 0) return fail(RMLX_E_BAD_ARG, "block_table_stride < 0");
  if (!aligned16(out_k) || !aligned16(out_v)) return fail(RMLX_E_BAD_ARG, "outputs must be 16-byte aligned");
  const int64_t out_layer_bytes = out_layer_stride * dtype_size(c.dtype);
  if (nl > 1 && (out_layer_stride <= 0 || out_layer_bytes % 16))
    return fail(RMLX_E_BAD_ARG, "out_layer_stride must be positive and a multiple of 16 bytes");
  DeviceGuard dg(p->device);
  cudaStream_t st = (cudaStream_t)stream;
  PoolGeo g = p->geo();
  const size_t smem = (size_t)(nseq + 1) * 2 * sizeof(int32_t);
  rmlx_status s;
  const bool fresh = p->gather_grid == 0 || p->gather_smem != smem;
  if (c.quant_bits == 0) {
    if (fresh) {
      if ((s = prepare_smem(gather_rows_kernel, smem)) != RMLX_OK) return s;
      p->gather_grid = persistent_grid(gather_rows_kernel, 256, smem, p->num_sms);
      p->gather_smem = smem;
    }
    cudaError_t e = launch_pdl(gather_rows_kernel, dim3(p->gather_grid), dim3(256), smem, st, g, layer, nl, bt,
                               bt_stride, lens, nseq, (uint8_t*)out_k, (uint8_t*)out_v, nl > 1 ? out_layer_bytes : 0,
                               p->err);
    if (e != cudaSuccess) return cuda_check(e, "gather launch");
  } else {
    const int ept = c.dtype == RMLX_F32 ? 4 : 8;  // output elements per 16-byte task
    const int tpr = c.head_dim / ept;
    const int idx = !is_pow2(tpr) ? 0 : (tpr <= 32 ? 2 : 1);
    const bool one_round = idx == 2 && (int64_t)c.block_size * tpr <= 256;  // 32 lanes x 8 tasks
    GatherDqFn fn = one_round ? pick_gather_dequant_r1(c.quant_bits, c.dtype, c.meta_dtype == RMLX_F32)
                              : pick_gather_dequant(c.quant_bits, c.dtype, c.meta_dtype == RMLX_F32, idx);
    if (fresh) {
      if ((s = prepare_smem(fn, smem)) != RMLX_OK) return s;
      p->gather_grid = persistent_grid(fn, 256, smem, p->num_sms);
      p->gather_smem = smem;
    }
    // one launch per layer (the dequantising kernels take one layer)
    for (int32_t i = 0; i < nl; ++i) {
      cudaError_t e = launch_pdl(fn, dim3(p->gather_grid), dim3(256), smem, st, g, layer + i, bt, bt_stride, lens,
                                 nseq, (uint8_t*)out_k + i * out_layer_bytes, (uint8_t*)out_v + i * out_layer_bytes,
                                 (int)c.head_dim, log2i(c.group_size), is_pow2(tpr) ? log2i(tpr) : -1, p->err);
      if (e != cudaSuccess) return cuda_check(e, "gather launch");
    }
  }
  return cuda_check(cudaGetLastError(), "gather launch");
}

rmlx_status rmlx_kv_gather(rmlx_kv_pool* p, int32_t layer, const int32_t* bt, int32_t bt_stride, const int32_t* lens,
                           int32_t nseq, void* out_k, void* out_v, void* stream) {
  if (p && (layer < 0 || layer >= p->cfg.num_layers))
    return fail(RMLX_E_RANGE, "layer %d outside the pool's %d layers", layer, p->cfg.num_layers);
  return gather_impl(p, layer, 1, bt, bt_stride, lens, nseq, out_k, out_v, 0, stream);
}

rmlx_status rmlx_kv_gather_layers(rmlx_kv_pool* p, int32_t layer_begin, int32_t num_layers, const int32_t* bt,
                                  int32_t bt_stride, const int32_t* lens, int32_t nseq, void* out_k, void* out_v,
                                  int64_t out_layer_stride, void* stream) {
  return gather_impl(p, layer_begin, num_layers, bt, bt_stride, lens, nseq, out_k, out_v, out_layer_stride, stream);
}

static rmlx_status launch_copy(rmlx_kv_pool* p, const int32_t* a, const int32_t* b, int32_t n, int mode,
                               uint8_t* staging, void* stream) {
  if (!p) return fail(RMLX_E_BAD_ARG, "NULL pool");
  if (n < 0) return fail(RMLX_E_BAD_ARG, "n < 0");
  if (n == 0) return RMLX_OK;
  if (!a || (mode == 0 && !b) || (mode != 0 && !staging)) return fail(RMLX_E_BAD_ARG, "NULL id array or staging");
  if (mode != 0 && !aligned16(staging)) return fail(RMLX_E_BAD_ARG, "staging must be 16-byte aligned");
  DeviceGuard dg(p->device);
  const int64_t units = (int64_t)n * (((int64_t)p->block_bytes + 4095) / 4096);
  const int grid = (int)std::min<int64_t>((units + 15) / 16, (int64_t)p->num_sms * 2);
  cudaError_t e = launch_pdl(copy_blocks_kernel, dim3(grid), dim3(256), 0, (cudaStream_t)stream, p->base,
                             (int64_t)p->block_bytes, (int)p->cfg.num_blocks, a, b, n, mode, staging, p->err);
  if (e != cudaSuccess) return cuda_check(e, "copy_blocks launch");
  return cuda_check(cudaGetLastError(), "copy_blocks launch");
}

rmlx_status rmlx_kv_copy_blocks(rmlx_kv_pool* p, const int32_t* src, const int32_t* dst, int32_t n, void* stream) {
  return launch_copy(p, src, dst, n, 0, nullptr, stream);
}
rmlx_status rmlx_kv_pack_blocks(rmlx_kv_pool* p, const int32_t* ids, int32_t n, void* staging, void* stream) {
  return launch_copy(p, ids, nullptr, n, 1, (uint8_t*)staging, stream);
}
rmlx_status rmlx_kv_unpack_blocks(rmlx_kv_pool* p, const int32_t* ids, int32_t n, const void* staging, void* stream) {
  return launch_copy(p, ids, nullptr, n, 2, (uint8_t*)staging, stream);
}

}  // extern "C"
