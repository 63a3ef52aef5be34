// widen.cuh -- exact widening of the weight formats to f16 pairs, for the
// tensor-core kernels that multiply half activations on kind::f16.
//
// int8 and E4M3 values are exact in f16; E2M1 times a power of two is exact
// as long as the product stays inside f16's range, which callers keep by a
// per-row exponent offset (see f16x2_pow2).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace mlpg {

// f16 multiplier 2^e for the E2M1 widening (e clamped to the f16 range).
__device__ __forceinline__ uint32_t f16x2_pow2(int e) {
  uint32_t h;
  if (e >= -14) h = (uint32_t)(min(e, 15) + 15) << 10;
  else if (e >= -24) h = 1u << (e + 24);
  else h = 0;
  return h | (h << 16);
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// 8 int8 (two words) -> 8 f16: bias to unsigned, place each byte under the
// exponent of 1024 (0x64xx = 1024 + byte), subtract 1152 (= 1024 + 128).
__device__ __forceinline__ uint4 widen_i8x8(uint2 v) {
  const uint32_t a = v.x ^ 0x80808080u, b = v.y ^ 0x80808080u;
  const uint32_t k = 0x64806480u;   // 1152.0 in both halves
  uint4 o;
  o.x = hsub2_u32(__byte_perm(a, 0x64646464u, 0x4140), k);
  o.y = hsub2_u32(__byte_perm(a, 0x64646464u, 0x4342), k);
  o.z = hsub2_u32(__byte_perm(b, 0x64646464u, 0x4140), k);
  o.w = hsub2_u32(__byte_perm(b, 0x64646464u, 0x4342), k);
  return o;
}

__device__ __forceinline__ uint32_t cvt_e4m3x2(uint32_t two_bytes) {
  uint32_t d;
  const unsigned short h = (unsigned short)two_bytes;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(h));
  return d;
}

__device__ __forceinline__ uint4 widen_e4m3x8(uint2 v) {
  uint4 o;
  o.x = cvt_e4m3x2(v.x);
  o.y = cvt_e4m3x2(v.x >> 16);
  o.z = cvt_e4m3x2(v.y);
  o.w = cvt_e4m3x2(v.y >> 16);
  return o;
}

// 8 E2M1 (one word, low nibble first) -> 4 f16 pairs, unscaled (exact).
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// 8 E2M1 (one word, low nibble first) -> 8 f16, times the f16x2 multiplier.
__device__ __forceinline__ uint4 widen_e2m1x8(uint32_t w, uint32_t mul) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
  return make_uint4(hmul2_u32(h0, mul), hmul2_u32(h1, mul), hmul2_u32(h2, mul), hmul2_u32(h3, mul));
}

}  // namespace mlpg
