// formats.cuh -- device decoders for the bench's number formats.
//
// Semantics follow the reference's host decoders (main.swift:30-48, :69-78):
//   E4M3  1-4-3, bias 7, exponent 0 -> m * 2^-9, 0x7F / 0xFF -> NaN
//   E2M1  1-2-1, bias 1, magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}
//   UE8M0 2^(code - 127)
// The decoders are exact: each places the format's exponent and mantissa
// bits into an IEEE float at a fixed offset and multiplies by the power of
// two that re-biases the exponent (subnormal inputs map to subnormal floats,
// so this relies on denormals being kept: the library is built without
// --use_fast_math / -ftz).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace mlpg {

// dtype codes (order of enum DType, main.swift:85-95)
enum DType : int {
  kFP16 = 0, kINT8 = 1, kI8I8 = 2, kFP8 = 3, kF8F8 = 4,
  kF4F4 = 5, kMXFP4 = 6, kMX4X4 = 7, kMX8X4 = 8, kF8X4 = 9, kNumDTypes = 10
};

__device__ __forceinline__ float dec_e4m3(uint32_t b) {
  // bits 6..0 (eeeemmm) -> f32 bits 26..20: value * 2^-120, rescale by 2^120.
  if ((b & 0x7Fu) == 0x7Fu) return __int_as_float(0x7FC00000);
  const float mag = __uint_as_float((b & 0x7Fu) << 20) * 1.329227995784916e36f;  // 2^120
  return (b & 0x80u) ? -mag : mag;
}

__device__ __forceinline__ float dec_e2m1(uint32_t n) {
  // bits 2..0 (eem) -> f32 bits 24..22: value * 2^-126, rescale by 2^126.
  const float mag = __uint_as_float((n & 7u) << 22) * 8.507059173023462e37f;  // 2^126
  return (n & 8u) ? -mag : mag;
}

__device__ __forceinline__ float dec_ue8m0(uint32_t c) {
  // 2^(c-127): c >= 1 is a normal float with exponent field c; c == 0 is 2^-127.
  return c ? __uint_as_float(c << 23) : __uint_as_float(0x00400000u);
}

__device__ __forceinline__ float dec_f16(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// Bytes per stored element of X / W for each dtype (FP4 = 1/2: "packed").
__host__ __device__ constexpr bool x_is_half(int dt) {
  return dt == kFP16 || dt == kINT8 || dt == kFP8 || dt == kMXFP4;
}
__host__ __device__ constexpr bool x_is_fp4(int dt) { return dt == kF4F4 || dt == kMX4X4; }
__host__ __device__ constexpr bool x_is_e4m3(int dt) {
  return dt == kF8F8 || dt == kMX8X4 || dt == kF8X4;
}
__host__ __device__ constexpr bool x_scaled(int dt) { return dt == kMX4X4 || dt == kMX8X4; }
__host__ __device__ constexpr bool w_is_mx(int dt) {
  return dt == kMXFP4 || dt == kMX4X4 || dt == kMX8X4 || dt == kF8X4;
}
__host__ __device__ constexpr bool w_is_half(int dt) { return dt == kFP16; }
__host__ __device__ constexpr bool w_is_i8(int dt) { return dt == kINT8 || dt == kI8I8; }
__host__ __device__ constexpr bool w_is_e4m3(int dt) { return dt == kFP8 || dt == kF8F8; }

// Decoded activation x[n,k] (refActivation, main.swift:419-436).
template <int DT>
__device__ __forceinline__ float load_x(const void* X, const uint8_t* xscale, int n, int k,
                                        int K) {
  const size_t i = (size_t)n * K + k;
  float v;
  if constexpr (x_is_half(DT)) {
    v = dec_f16(reinterpret_cast<const uint16_t*>(X)[i]);
  } else if constexpr (DT == kI8I8) {
    v = (float)reinterpret_cast<const int8_t*>(X)[i];
  } else if constexpr (x_is_e4m3(DT)) {
    v = dec_e4m3(reinterpret_cast<const uint8_t*>(X)[i]);
  } else {  // FP4, low nibble = even element
    const uint8_t b = reinterpret_cast<const uint8_t*>(X)[i >> 1];
    v = dec_e2m1((i & 1) ? (b >> 4) : (b & 0xF));
  }
  if constexpr (x_scaled(DT)) {
    v *= dec_ue8m0(xscale[(size_t)n * (K / 32) + k / 32]);
  }
  return v;
}

}  // namespace mlpg
