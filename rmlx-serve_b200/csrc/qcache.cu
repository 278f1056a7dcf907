// Device-backed QuantizedKVCache: the drop-in for
// crates/rmlx-serve-cache/src/quantized_cache.rs:14-296.
//
// Keeps the reference's host-slice API and its exact storage: per layer, a
// flat byte stream plus per-group f32 scales and zeros, appended in call
// order; each append slices its [heads, tokens, head_dim] f32 input into
// groups of group_size (a trailing partial group allowed, :177-197).  The
// bytes, scales and zeros live in device memory; quantisation and
// dequantisation run as one warp per group.  Dequantisation reproduces
// dequantize_data (:200-223) including its reading frame: group g reads
// bytes [g * bytes_per_group, ...) whatever the appends stored, and a group
// that starts past the end is the reference's slice panic (RMLX_E_BAD_ARG).
#include <mutex>
#include <new>
#include <vector>

#include "device_common.cuh"

namespace rmlx {

__device__ __forceinline__ uint32_t qcode(float v, float mn, float scale, float qmax) {
  float x = roundf(__fdiv_rn(__fsub_rn(v, mn), scale));
  if (x < 0.0f) x = 0.0f;
  if (x > qmax) x = qmax;
  return (x == x) ? (uint32_t)x : 0u;
}

// quantize_group (:232-273) for every group of one append.
template <int BITS>
__global__ void qcache_quant_kernel(const float* __restrict__ in, int64_t n, int gs, int ng, uint8_t* out_bytes,
                                    float* scales, float* zeros) {
  const int lane = threadIdx.x & 31;
  const int64_t g = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (g >= ng) return;
  const int64_t s = g * gs;
  const int len = (int)min((int64_t)gs, n - s);
  float mx = -INFINITY, mn = INFINITY;
  for (int i = lane; i < len; i += 32) {
    float x = in[s + i];
    mx = fmaxf(mx, x);
    mn = fminf(mn, x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
  }
  const float qmax = (float)((1u << BITS) - 1);
  const float range = __fsub_rn(mx, mn);
  const float scale = range == 0.0f ? 1.0f : __fdiv_rn(range, qmax);
  if (BITS == 8) {
    uint8_t* o = out_bytes + g * gs;
    for (int i = lane; i < len; i += 32) o[i] = (uint8_t)qcode(in[s + i], mn, scale, qmax);
  } else {
    uint8_t* o = out_bytes + g * ((gs + 1) / 2);
    for (int j = lane; j < (len + 1) / 2; j += 32) {
      uint32_t lo = qcode(in[s + 2 * j], mn, scale, qmax);
      uint32_t hi = (2 * j + 1 < len) ? qcode(in[s + 2 * j + 1], mn, scale, qmax) : 0u;
      o[j] = (uint8_t)(lo | (hi << 4));
    }
  }
  if (lane == 0) {
    scales[g] = scale;
    zeros[g] = mn;
  }
}

// dequantize_group (:278-296) over the reading frame of dequantize_data.
template <int BITS>
__global__ void qcache_dequant_kernel(const uint8_t* __restrict__ bytes, int64_t nbytes, int bpg, int ng,
                                      const float* __restrict__ scales, const float* __restrict__ zeros, float* out) {
  const int lane = threadIdx.x & 31;
  const int64_t g = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (g >= ng) return;
  const int64_t b0 = g * bpg;
  const int64_t b1 = min(b0 + bpg, nbytes);
  const float sc = scales[g], zr = zeros[g];
  if (BITS == 8) {
    float* o = out + b0;
    for (int64_t i = lane; i < b1 - b0; i += 32) o[i] = __fadd_rn(__fmul_rn((float)bytes[b0 + i], sc), zr);
  } else {
    float* o = out + 2 * b0;
    for (int64_t i = lane; i < b1 - b0; i += 32) {
      uint32_t b = bytes[b0 + i];
      o[2 * i] = __fadd_rn(__fmul_rn((float)(b & 0xFu), sc), zr);
      o[2 * i + 1] = __fadd_rn(__fmul_rn((float)((b >> 4) & 0xFu), sc), zr);
    }
  }
}

template <typename T>
struct DevVec {
  T* ptr = nullptr;
  size_t len = 0, cap = 0;
  rmlx_status reserve(size_t need) {
    if (need <= cap) return RMLX_OK;
    size_t nc = cap ? cap : 256;
    while (nc < need) nc *= 2;
    T* np = nullptr;
    if (cudaMalloc(&np, nc * sizeof(T)) != cudaSuccess) {
      cudaGetLastError();
      return fail(RMLX_E_EXHAUSTED, "cudaMalloc(%zu bytes) failed", nc * sizeof(T));
    }
    if (len) {
      rmlx_status s = cuda_check(cudaMemcpy(np, ptr, len * sizeof(T), cudaMemcpyDeviceToDevice), "grow copy");
      if (s != RMLX_OK) {
        cudaFree(np);
        return s;
      }
    }
    cudaFree(ptr);
    ptr = np;
    cap = nc;
    return RMLX_OK;
  }
  void release() {
    cudaFree(ptr);
    ptr = nullptr;
    len = cap = 0;
  }
};

struct QLayer {
  DevVec<uint8_t> bytes;
  DevVec<float> scales, zeros;
};

}  // namespace rmlx

using namespace rmlx;

struct rmlx_qcache {
  size_t layers, heads, hd, bits, gs;
  int device;
  size_t seq_len = 0;
  std::vector<QLayer> k, v;
  DevVec<float> stage_in, stage_out;
};

namespace {

rmlx_status quantize_into(rmlx_qcache* q, QLayer& L, const float* dev_in, size_t n) {
  const size_t ng = (n + q->gs - 1) / q->gs;
  const size_t bpg = q->bits == 4 ? (q->gs + 1) / 2 : q->gs;
  // Bytes this call adds: full groups are bpg each, the last holds the rest.
  const size_t last = n - (ng - 1) * q->gs;
  const size_t add = (ng - 1) * bpg + (q->bits == 4 ? (last + 1) / 2 : last);
  rmlx_status s;
  if ((s = L.bytes.reserve(L.bytes.len + add)) != RMLX_OK) return s;
  if ((s = L.scales.reserve(L.scales.len + ng)) != RMLX_OK) return s;
  if ((s = L.zeros.reserve(L.zeros.len + ng)) != RMLX_OK) return s;
  const int grid = (int)((ng * 32 + 255) / 256);
  if (q->bits == 8)
    qcache_quant_kernel<8><<<grid, 256>>>(dev_in, (int64_t)n, (int)q->gs, (int)ng, L.bytes.ptr + L.bytes.len,
                                          L.scales.ptr + L.scales.len, L.zeros.ptr + L.zeros.len);
  else
    qcache_quant_kernel<4><<<grid, 256>>>(dev_in, (int64_t)n, (int)q->gs, (int)ng, L.bytes.ptr + L.bytes.len,
                                          L.scales.ptr + L.scales.len, L.zeros.ptr + L.zeros.len);
  if ((s = cuda_check(cudaGetLastError(), "qcache quant launch")) != RMLX_OK) return s;
  L.bytes.len += add;
  L.scales.len += ng;
  L.zeros.len += ng;
  return RMLX_OK;
}

rmlx_status dequantize_layer(rmlx_qcache* q, QLayer& L, float* out, size_t cap, size_t* n_out) {
  *n_out = 0;
  if (L.bytes.len == 0) return RMLX_OK;  // quantized_cache.rs:201-203
  const size_t bpg = q->bits == 4 ? (q->gs + 1) / 2 : q->gs;
  const size_t vpb = q->bits == 4 ? 2 : 1;
  const size_t ng = L.scales.len;
  if (ng == 0) return RMLX_OK;
  if ((ng - 1) * bpg > L.bytes.len)
    return fail(RMLX_E_BAD_ARG, "group %zu starts past the %zu stored bytes (slice out of range)", ng - 1, L.bytes.len);
  const size_t n = ((ng - 1) * bpg + std::min(bpg, L.bytes.len - (ng - 1) * bpg)) * vpb;
  *n_out = n;
  if (!out) return RMLX_OK;
  if (cap < n) return fail(RMLX_E_BAD_ARG, "output holds %zu floats, %zu needed", cap, n);
  DeviceGuard dg(q->device);
  rmlx_status s;
  if ((s = q->stage_out.reserve(n)) != RMLX_OK) return s;
  const int grid = (int)((ng * 32 + 255) / 256);
  if (q->bits == 8)
    qcache_dequant_kernel<8><<<grid, 256>>>(L.bytes.ptr, (int64_t)L.bytes.len, (int)bpg, (int)ng, L.scales.ptr,
                                            L.zeros.ptr, q->stage_out.ptr);
  else
    qcache_dequant_kernel<4><<<grid, 256>>>(L.bytes.ptr, (int64_t)L.bytes.len, (int)bpg, (int)ng, L.scales.ptr,
                                            L.zeros.ptr, q->stage_out.ptr);
  if ((s = cuda_check(cudaGetLastError(), "qcache dequant launch")) != RMLX_OK) return s;
  return cuda_check(cudaMemcpy(out, q->stage_out.ptr, n * sizeof(float), cudaMemcpyDeviceToHost), "dequant copy-out");
}

}  // namespace

// ---------------------------------------------------------------------------
// Dequantise through a fixed device array instead of allocated scratch.
//
// Some callers cannot call cudaMalloc while they run: a serving engine that
// gave nearly all free GPU memory to its KV pool at start-up (rmlx-serve's
// CacheConfig defaults gpu_memory_utilization to 0.9) may see a later
// allocation fail or eat into memory it already promised the pool, and code
// on the per-step path cannot afford the device-wide synchronisation that
// cudaMalloc/cudaFree may cause.  rmlx_qcache_get_dequantized_static serves
// them: it stages the dequantised values in g_static_dequant, a file-scope
// device array that exists on every GPU that loads this library, for as long
// as the process runs, and it calls no allocator.
//
// In host code `g_static_dequant` names a host-side stand-in, not device
// memory, so the device address is looked up once per device (with that
// device current) and cached in g_static_addr.  Every call shares the one
// array per device and leaves its values there; the kernel overwrites every
// value a call copies out, so nothing needs clearing between calls, but two
// calls whose work overlaps on the same GPU race on the array.
// ---------------------------------------------------------------------------
static constexpr size_t kStaticMaxFloats = RMLX_QCACHE_STATIC_MAX_FLOATS;
static __device__ __align__(256) float g_static_dequant[kStaticMaxFloats];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
float* g_static_addr[kMaxDevices] = {};

// Device address of g_static_dequant on `device` (already current).
rmlx_status static_scratch(int device, float** out) {
  if (device < 0 || device >= kMaxDevices) return fail(RMLX_E_BAD_ARG, "device %d out of range", device);
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_addr[device]) {
    void* p = nullptr;
    rmlx_status s = cuda_check(cudaGetSymbolAddress(&p, g_static_dequant), "cudaGetSymbolAddress(static scratch)");
    if (s != RMLX_OK) return s;
    g_static_addr[device] = static_cast<float*>(p);
  }
  *out = g_static_addr[device];
  return RMLX_OK;
}
}  // namespace

extern "C" rmlx_status rmlx_qcache_get_dequantized_static(rmlx_qcache* q, size_t layer, int32_t which, float* out,
                                                          size_t cap, size_t* n_out) {
  if (!q || !n_out) return fail(RMLX_E_BAD_ARG, "NULL cache or n_out");
  if (layer >= q->layers) return fail(RMLX_E_RANGE, "layer %zu out of range", layer);
  if (which != 0 && which != 1) return fail(RMLX_E_BAD_ARG, "which must be 0 (keys) or 1 (values)");
  QLayer& L = which ? q->v[layer] : q->k[layer];
  *n_out = 0;
  if (L.bytes.len == 0 || L.scales.len == 0) return RMLX_OK;
  const size_t bpg = q->bits == 4 ? (q->gs + 1) / 2 : q->gs;
  const size_t vpb = q->bits == 4 ? 2 : 1;
  const size_t ng = L.scales.len;
  if ((ng - 1) * bpg > L.bytes.len)
    return fail(RMLX_E_BAD_ARG, "group %zu starts past the %zu stored bytes (slice out of range)", ng - 1, L.bytes.len);
  const size_t n = ((ng - 1) * bpg + std::min(bpg, L.bytes.len - (ng - 1) * bpg)) * vpb;
  *n_out = n;
  if (!out) return RMLX_OK;
  if (n > kStaticMaxFloats)
    return fail(RMLX_E_BAD_ARG, "%zu values exceed the static scratch of %zu floats", n, kStaticMaxFloats);
  if (cap < n) return fail(RMLX_E_BAD_ARG, "output holds %zu floats, %zu needed", cap, n);
  DeviceGuard dg(q->device);
  float* scratch = nullptr;
  rmlx_status s = static_scratch(q->device, &scratch);
  if (s != RMLX_OK) return s;
  const int grid = (int)((ng * 32 + 255) / 256);
  if (q->bits == 8)
    qcache_dequant_kernel<8><<<grid, 256>>>(L.bytes.ptr, (int64_t)L.bytes.len, (int)bpg, (int)ng, L.scales.ptr,
                                            L.zeros.ptr, scratch);
  else
    qcache_dequant_kernel<4><<<grid, 256>>>(L.bytes.ptr, (int64_t)L.bytes.len, (int)bpg, (int)ng, L.scales.ptr,
                                            L.zeros.ptr, scratch);
  if ((s = cuda_check(cudaGetLastError(), "static dequant launch")) != RMLX_OK) return s;
  return cuda_check(cudaMemcpy(out, scratch, n * sizeof(float), cudaMemcpyDeviceToHost), "static dequant copy-out");
}

extern "C" {

rmlx_status rmlx_qcache_new(size_t num_layers, size_t num_kv_heads, size_t head_dim, size_t bits, size_t group_size,
                            int device, rmlx_qcache** out) {
  if (!out) return fail(RMLX_E_BAD_ARG, "out is NULL");
  *out = nullptr;
  if (bits != 4 && bits != 8) return fail(RMLX_E_BAD_ARG, "bits must be 4 or 8, got %zu", bits);  // :57-60
  if (group_size == 0) return fail(RMLX_E_BAD_ARG, "group_size must be > 0");
  if (!(head_dim % group_size == 0 || group_size > head_dim))  // :61-65
    return fail(RMLX_E_BAD_ARG, "head_dim (%zu) should be divisible by group_size (%zu)", head_dim, group_size);
  rmlx_qcache* q = new (std::nothrow) rmlx_qcache();
  if (!q) return fail(RMLX_E_EXHAUSTED, "host allocation failed");
  q->layers = num_layers;
  q->heads = num_kv_heads;
  q->hd = head_dim;
  q->bits = bits;
  q->gs = group_size;
  q->device = device;
  q->k.resize(num_layers);
  q->v.resize(num_layers);
  *out = q;
  return RMLX_OK;
}

void rmlx_qcache_destroy(rmlx_qcache* q) {
  if (!q) return;
  {
    DeviceGuard dg(q->device);
    for (auto* side : {&q->k, &q->v})
      for (auto& L : *side) {
        L.bytes.release();
        L.scales.release();
        L.zeros.release();
      }
    q->stage_in.release();
    q->stage_out.release();
  }
  delete q;
}

rmlx_status rmlx_qcache_append(rmlx_qcache* q, size_t layer, const float* keys, const float* values, size_t len,
                               size_t new_tokens) {
  if (!q) return fail(RMLX_E_BAD_ARG, "NULL cache");
  if (layer >= q->layers) return fail(RMLX_E_RANGE, "layer %zu out of range (%zu layers)", layer, q->layers);
  const size_t expected = q->heads * new_tokens * q->hd;
  if (len != expected)  // :96-108
    return fail(RMLX_E_BAD_ARG, "keys length mismatch: expected %zu, got %zu", expected, len);
  if (len > 0) {
    if (!keys || !values) return fail(RMLX_E_BAD_ARG, "NULL keys or values");
    DeviceGuard dg(q->device);
    rmlx_status s;
    if ((s = q->stage_in.reserve(2 * len)) != RMLX_OK) return s;
    float* dk = q->stage_in.ptr;
    float* dv = q->stage_in.ptr + len;
    if ((s = cuda_check(cudaMemcpy(dk, keys, len * sizeof(float), cudaMemcpyHostToDevice), "keys H2D")) != RMLX_OK ||
        (s = cuda_check(cudaMemcpy(dv, values, len * sizeof(float), cudaMemcpyHostToDevice), "values H2D")) != RMLX_OK)
      return s;
    if ((s = quantize_into(q, q->k[layer], dk, len)) != RMLX_OK) return s;
    if ((s = quantize_into(q, q->v[layer], dv, len)) != RMLX_OK) return s;
    if ((s = cuda_check(cudaDeviceSynchronize(), "qcache append")) != RMLX_OK) return s;
  }
  if (layer == 0) q->seq_len += new_tokens;  // :124-126
  return RMLX_OK;
}

rmlx_status rmlx_qcache_get_keys_dequantized(rmlx_qcache* q, size_t layer, float* out, size_t cap, size_t* n_out) {
  if (!q || !n_out) return fail(RMLX_E_BAD_ARG, "NULL cache or n_out");
  if (layer >= q->layers) return fail(RMLX_E_RANGE, "layer %zu out of range", layer);
  return dequantize_layer(q, q->k[layer], out, cap, n_out);
}
rmlx_status rmlx_qcache_get_values_dequantized(rmlx_qcache* q, size_t layer, float* out, size_t cap, size_t* n_out) {
  if (!q || !n_out) return fail(RMLX_E_BAD_ARG, "NULL cache or n_out");
  if (layer >= q->layers) return fail(RMLX_E_RANGE, "layer %zu out of range", layer);
  return dequantize_layer(q, q->v[layer], out, cap, n_out);
}
size_t rmlx_qcache_seq_len(const rmlx_qcache* q) { return q->seq_len; }
size_t rmlx_qcache_num_layers(const rmlx_qcache* q) { return q->layers; }
size_t rmlx_qcache_bits(const rmlx_qcache* q) { return q->bits; }
size_t rmlx_qcache_group_size(const rmlx_qcache* q) { return q->gs; }

rmlx_status rmlx_qcache_raw(rmlx_qcache* q, size_t layer, int32_t which, uint8_t* bytes, size_t bcap, float* sc,
                            float* zr, size_t gcap, size_t* n_bytes, size_t* n_groups) {
  if (!q || !n_bytes || !n_groups) return fail(RMLX_E_BAD_ARG, "NULL argument");
  if (layer >= q->layers) return fail(RMLX_E_RANGE, "layer %zu out of range", layer);
  if (which != 0 && which != 1) return fail(RMLX_E_BAD_ARG, "which must be 0 (keys) or 1 (values)");
  QLayer& L = which ? q->v[layer] : q->k[layer];
  *n_bytes = L.bytes.len;
  *n_groups = L.scales.len;
  DeviceGuard dg(q->device);
  rmlx_status s;
  size_t nb = std::min(bcap, L.bytes.len), ng = std::min(gcap, L.scales.len);
  if (bytes && nb &&
      (s = cuda_check(cudaMemcpy(bytes, L.bytes.ptr, nb, cudaMemcpyDeviceToHost), "raw bytes")) != RMLX_OK)
    return s;
  if (sc && ng &&
      (s = cuda_check(cudaMemcpy(sc, L.scales.ptr, ng * sizeof(float), cudaMemcpyDeviceToHost), "raw scales")) != RMLX_OK)
    return s;
  if (zr && ng &&
      (s = cuda_check(cudaMemcpy(zr, L.zeros.ptr, ng * sizeof(float), cudaMemcpyDeviceToHost), "raw zeros")) != RMLX_OK)
    return s;
  return RMLX_OK;
}

}  // extern "C"
