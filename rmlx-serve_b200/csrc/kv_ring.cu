// Rotating (sliding-window) cache as a ring over a sequence's blocks
// (RotatingKVCache, crates/rmlx-serve-cache/src/rotating_cache.rs:94-262).
//
// A ring sequence of max_size rows keeps its first `keep` rows and cycles
// the other R = max_size - keep through ring positions keep .. max_size-1;
// ring position p lives in block table entry p / block_size, row
// p % block_size.  The host keeps the reference's (written, offset) state
// and turns each append into slot mappings for rmlx_kv_append.  On the
// device this file adds:
//   * gather in logical order (get_logical_order, :162-197): logical row i
//     of a sequence is ring position i while nothing has rotated, else i for
//     i < keep and keep + (offset + i - keep) % R after;
//   * a row move (the data shift of trim before rotation, :213-247), staged
//     through a scratch buffer so that overlapping source and destination
//     ranges move as one copy.
#include <algorithm>

#include "kv_pool_internal.cuh"

namespace rmlx {

// One warp per (sequence, kv, head, 16 logical rows); lanes stream the rows'
// 16-byte chunks.  ring_offset[s] < 0: no rotation (identity order).
__global__ void __launch_bounds__(256) gather_ring_kernel(PoolGeo g, int layer, const int32_t* __restrict__ bt,
                                                          int bt_stride, const int32_t* __restrict__ lens,
                                                          const int32_t* __restrict__ ring_offset, int nseq, int keep,
                                                          int ring, uint8_t* __restrict__ ok, uint8_t* __restrict__ ov,
                                                          int32_t* err) {
  constexpr int ROWS = 16;
  extern __shared__ int32_t smem[];
  int32_t* cub = smem;
  int32_t* cut = smem + nseq + 1;
  pdl_wait();
  pdl_release();
  scan_seq_lens(lens, nseq, ROWS, cub, cut);
  const int64_t units = (int64_t)cub[nseq] * 2 * g.heads;
  const int lane = threadIdx.x & 31;
  const int cpr = g.row_bytes / 16;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t u = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < units; u += nwarps) {
    const int h = (int)(u % g.heads);
    const int64_t q = u / g.heads;
    const int kv = (int)(q & 1);
    const int64_t gi = q >> 1;
    const int s = find_seq(cub, nseq, gi);
    const int c = (int)(gi - cub[s]);
    const int L = cut[s + 1] - cut[s];
    const int off = __ldg(ring_offset + s);
    uint8_t* out = (kv ? ov : ok) + ((int64_t)cut[s] * g.heads + (int64_t)h * L) * g.row_bytes;
    const int nrows = min(ROWS, L - c * ROWS);
    for (int idx = lane; idx < nrows * cpr; idx += 32) {
      const int r = idx / cpr, ch = idx - r * cpr;
      const int i = c * ROWS + r;  // logical row
      int p = i;
      if (off >= 0 && i >= keep) p = keep + (int)(((int64_t)off + (i - keep)) % ring);
      const int32_t blk = __ldg(bt + (int64_t)s * bt_stride + p / g.bs);
      if (blk < 0 || blk >= g.nblocks) {
        atomicOr(err, DEV_ERR_BLOCK);
        continue;
      }
      const uint8_t* src = g.base + g.tile_off(blk, layer, kv, h) + (int64_t)(p % g.bs) * g.row_bytes + ch * 16;
      st_stream(out + (int64_t)i * g.row_bytes + ch * 16, ld_stream(src));
    }
  }
}

// Rows of slot src[i] <-> staging (dir 0: pool -> staging, 1: staging ->
// pool at slot dst[i]); all layers, K and V, every head, code and meta rows.
// Staging holds per moved row and (layer, kv, head): row_bytes, then the
// meta row padded to 16 bytes (so every 16-byte access stays aligned).
// Meta rows are copied in 4-byte words.
__global__ void __launch_bounds__(256) move_rows_kernel(PoolGeo g, const int32_t* __restrict__ slots, int n, int dir,
                                                        uint8_t* __restrict__ staging, int32_t* err) {
  pdl_wait();
  pdl_release();
  const int rb = g.row_bytes, mb = g.meta_row_bytes;
  const int per_tile = rb / 16 + mb / 4;  // copy units per (row, layer, kv, head)
  const int64_t tiles = (int64_t)g.layers * 2 * g.heads;
  const int64_t total = (int64_t)n * tiles * per_tile;
  const int sstride = rb + ((mb + 15) & ~15);
  const int64_t row_stage = tiles * sstride;
  const int64_t cap = (int64_t)g.nblocks * g.bs;
  for (int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; x < total; x += (int64_t)gridDim.x * blockDim.x) {
    const int w = (int)(x % per_tile);
    const int64_t t = (x / per_tile) % tiles;  // (layer, kv, head) flattened
    const int i = (int)(x / per_tile / tiles);
    const int32_t slot = __ldg(slots + i);
    if (slot < 0 || slot >= cap) {
      atomicOr(err, DEV_ERR_SLOT);
      continue;
    }
    const int blk = slot / g.bs, row = slot % g.bs;
    const int h = (int)(t % g.heads), kv = (int)((t / g.heads) & 1), l = (int)(t / g.heads / 2);
    uint8_t* tile = g.base + g.tile_off(blk, l, kv, h);
    uint8_t* st = staging + i * row_stage + t * sstride;
    if (w < rb / 16) {
      uint8_t* pr = tile + (int64_t)row * rb + w * 16;
      if (dir == 0) st_stream(st + w * 16, ld_stream(pr));
      else st_stream(pr, ld_stream(st + w * 16));
    } else {
      const int m = w - rb / 16;
      uint32_t* pm = reinterpret_cast<uint32_t*>(tile + (int64_t)g.bs * rb + (int64_t)row * mb) + m;
      uint32_t* sm = reinterpret_cast<uint32_t*>(st + rb) + m;
      if (dir == 0) *sm = *pm;
      else *pm = *sm;
    }
  }
}

}  // namespace rmlx

using namespace rmlx;

extern "C" {

rmlx_status rmlx_kv_gather_ring(rmlx_kv_pool* p, int32_t layer, const int32_t* block_tables, int32_t block_table_stride,
                                const int32_t* seq_lens, const int32_t* ring_offsets, int32_t num_seqs, int32_t keep,
                                int32_t max_size, void* out_k, void* out_v, void* stream) {
  if (!p) return fail(RMLX_E_BAD_ARG, "NULL pool");
  const rmlx_pool_config& c = p->cfg;
  if (c.quant_bits) return fail(RMLX_E_BAD_ARG, "ring gather reads unquantised pools");
  if (layer < 0 || layer >= c.num_layers) return fail(RMLX_E_RANGE, "layer %d out of range", layer);
  if (keep < 0 || keep >= max_size)
    return fail(RMLX_E_BAD_ARG, "keep (%d) must be less than max_size (%d)", keep, max_size);
  if (num_seqs < 0 || num_seqs > RMLX_MAX_SEQS_PER_LAUNCH) return fail(RMLX_E_BAD_ARG, "num_seqs out of range");
  if (num_seqs == 0) return RMLX_OK;
  if (!block_tables || !seq_lens || !ring_offsets || !out_k || !out_v) return fail(RMLX_E_BAD_ARG, "NULL argument");
  if (!aligned16(out_k) || !aligned16(out_v)) return fail(RMLX_E_BAD_ARG, "outputs must be 16-byte aligned");
  DeviceGuard dg(p->device);
  const size_t smem = (size_t)2 * (num_seqs + 1) * 4;
  rmlx_status s;
  if ((s = prepare_smem(gather_ring_kernel, smem)) != RMLX_OK) return s;
  const int grid = persistent_grid(gather_ring_kernel, 256, smem, p->num_sms);
  cudaError_t e = launch_pdl(gather_ring_kernel, dim3(grid), dim3(256), smem, (cudaStream_t)stream, p->geo(),
                             (int)layer, block_tables, (int)block_table_stride, seq_lens, ring_offsets, (int)num_seqs,
                             (int)keep, (int)(max_size - keep), (uint8_t*)out_k, (uint8_t*)out_v, p->err);
  if (e != cudaSuccess) return cuda_check(e, "ring gather launch");
  return cuda_check(cudaGetLastError(), "ring gather launch");
}

rmlx_status rmlx_kv_move_rows(rmlx_kv_pool* p, const int32_t* src_slots, const int32_t* dst_slots, int32_t n,
                              void* stream) {
  if (!p) return fail(RMLX_E_BAD_ARG, "NULL pool");
  if (n < 0) return fail(RMLX_E_BAD_ARG, "n < 0");
  if (n == 0) return RMLX_OK;
  if (!src_slots || !dst_slots) return fail(RMLX_E_BAD_ARG, "NULL slots");
  DeviceGuard dg(p->device);
  cudaStream_t st = (cudaStream_t)stream;
  const PoolGeo g = p->geo();
  const int64_t tiles = (int64_t)g.layers * 2 * g.heads;
  const size_t bytes = (size_t)n * tiles * (g.row_bytes + ((g.meta_row_bytes + 15) & ~15));
  void* staging = nullptr;
  if (cudaMallocAsync(&staging, bytes, st) != cudaSuccess) return cuda_check(cudaGetLastError(), "move_rows staging");
  const int64_t total = (int64_t)n * tiles * (g.row_bytes / 16 + g.meta_row_bytes / 4);
  const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)p->num_sms * 8);
  cudaError_t e = launch_pdl(move_rows_kernel, dim3(grid), dim3(256), 0, st, g, src_slots, (int)n, 0,
                             (uint8_t*)staging, p->err);
  if (e == cudaSuccess)
    e = launch_pdl(move_rows_kernel, dim3(grid), dim3(256), 0, st, g, dst_slots, (int)n, 1, (uint8_t*)staging, p->err);
  cudaFreeAsync(staging, st);
  if (e != cudaSuccess) return cuda_check(e, "move_rows launch");
  return cuda_check(cudaGetLastError(), "move_rows launch");
}

}  // extern "C"
