// Group-affine dequantisation of one code, shared by the dequantise-on-
// gather kernels (kv_pool.cu) and the decode attention over quantised pools
// (kv_attention.cu), so both see the same values: (code as f32) * scale +
// zero as dequantize_group computes it (quantized_cache.rs:278-296), rounded
// once per step, then rounded to the output type by the caller.
//
// The code's f32 value comes from a byte permute that builds the bit pattern
// of 2^23 + code (exact for codes < 2^23) and an exact subtraction of 2^23.
// With f32 scale/zero: a rounded multiply then a rounded add.  With f16
// scale/zero: code * scale is exact in f32 (a code has at most 8
// significant bits and an f16 value 11, and the product stays in f32's
// normal range), so one fused multiply-add (rounded once, after the add)
// gives the same value; the packed f32x2 forms do two elements at a time.
#pragma once
#include <cstdint>

namespace rmlx {

// f32 bit pattern of 2^23 + byte `b` of `w`.
__device__ __forceinline__ float magic_byte(uint32_t w, int b) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)b));
}

// Two f32 values in one 64-bit register, for the packed f32x2 instructions.
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f32x2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Dequantised elements e and e + 1 (e even) of a task.  8-bit: bytes of the
// task's code words; 4-bit: the low and high nibble of byte e / 2, taken
// from the pre-masked words lo4 (low nibbles) and hi4 (high nibbles).
template <int BITS, bool META_F32>
__device__ __forceinline__ void dq_pair(const uint2& cw, uint32_t lo4, uint32_t hi4, int e, float sc, float zr,
                                        float& a, float& b) {
  float m0, m1;
  if (BITS == 8) {
    const uint32_t w = e < 4 ? cw.x : cw.y;
    m0 = magic_byte(w, e & 3);
    m1 = magic_byte(w, (e + 1) & 3);
  } else {
    m0 = magic_byte(lo4, e >> 1);
    m1 = magic_byte(hi4, e >> 1);
  }
  if (META_F32) {
    a = __fadd_rn(__fmul_rn(__fadd_rn(m0, -8388608.0f), sc), zr);
    b = __fadd_rn(__fmul_rn(__fadd_rn(m1, -8388608.0f), sc), zr);
  } else {
    const uint64_t q = add_f32x2(f32x2(m0, m1), f32x2(-8388608.0f, -8388608.0f));
    f32x2_split(fma_f32x2(q, f32x2(sc, sc), f32x2(zr, zr)), a, b);
  }
}

}  // namespace rmlx
