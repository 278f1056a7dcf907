// Device-side helpers shared by the rmlx_kv CUDA sources (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

#include "common.h"

namespace rmlx {

// Error bits latched into a pool's device error word.
enum : int32_t {
  DEV_ERR_SLOT = 1,   // slot_mapping entry >= num_blocks * block_size
  DEV_ERR_BLOCK = 2,  // block-table / copy id outside [0, num_blocks)
  DEV_ERR_WORKSPACE = 4,  // a launch's splits exceed the workspace it was given
};

// 16-byte streaming load through the non-coherent path without L1
// allocation: every byte of the pool and of the inputs is read once per
// launch, so nothing is worth keeping in L1.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// 16-byte store with the evict-first (streaming) policy: gathered rows are
// consumed by the next kernel or copied out, not re-read by this one.
__device__ __forceinline__ void st_stream(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// A warp copies n16 16-byte chunks from src to dst, 8 chunks per lane in
// flight (4 KiB per warp per round).
__device__ __forceinline__ void warp_copy(const uint8_t* src, uint8_t* dst, int n16, int lane) {
  for (int base = 0; base < n16; base += 256) {
    uint4 r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int c = base + lane + 32 * j;
      if (c < n16) r[j] = ld_stream(src + (size_t)c * 16);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int c = base + lane + 32 * j;
      if (c < n16) st_stream(dst + (size_t)c * 16, r[j]);
    }
  }
}

// A warp copies two independent runs (n16a and n16b 16-byte chunks) with all
// of their loads issued before any store: up to 16 chunks (8 KiB per warp)
// in flight per round.  Two 4 KiB tiles per warp at two 256-thread CTAs per
// SM keep ~128 KiB of reads in flight per SM, which measured 6% faster on
// B200 than one tile per warp at four CTAs per SM.
__device__ __forceinline__ void warp_copy2(const uint8_t* sa, uint8_t* da, int n16a, const uint8_t* sb, uint8_t* db,
                                           int n16b, int lane) {
  const int n = n16a > n16b ? n16a : n16b;
  for (int base = 0; base < n; base += 256) {
    uint4 ra[8], rb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int c = base + lane + 32 * j;
      if (c < n16a) ra[j] = ld_stream(sa + (size_t)c * 16);
      if (c < n16b) rb[j] = ld_stream(sb + (size_t)c * 16);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int c = base + lane + 32 * j;
      if (c < n16a) st_stream(da + (size_t)c * 16, ra[j]);
      if (c < n16b) st_stream(db + (size_t)c * 16, rb[j]);
    }
  }
}

// Programmatic dependent launch.  Kernels are launched with programmatic
// stream serialisation, so the next kernel in the stream may be scheduled
// before this one finishes; pdl_wait() (at the top of every kernel, before
// any global memory access) blocks until the preceding grid has completed
// and its writes are visible, and pdl_release() lets the next grid start
// launching.  Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with programmatic stream serialisation (see pdl_wait).
template <typename... Exp, typename... Act>
cudaError_t launch_pdl(void (*kernel)(Exp...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Act&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Act>(args)...);
}

// RAII switch of the current device for the duration of an API call.
struct DeviceGuard {
  int prev = -1, dev;
  explicit DeviceGuard(int d) : dev(d) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0 && prev != dev) cudaSetDevice(prev);
  }
};

inline rmlx_status cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return RMLX_OK;
  return fail(RMLX_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace rmlx
