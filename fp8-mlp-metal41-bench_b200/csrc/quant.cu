// quant.cu -- the bench's wire formats produced from f32 on the device.
//
// The reference produces its operands on the host, untimed: floatToE4M3
// (main.swift:6-27), E2M1 codes packed two per byte with the low nibble the
// even element (main.swift:50-67), UE8M0 scale codes (main.swift:76-83).
// These kernels produce the same formats from f32 data on the GPU:
//
//   GEMM_Q_E4M3_REF  the reference encoder, bit for bit (round half up on the
//                    first dropped bit, flush below 2^-6, saturation to 0x7E)
//   GEMM_Q_E4M3      OCP E4M3FN: round to nearest even, subnormals, saturating
//                    at +-448 (cvt.rn.satfinite.e4m3x2.f32); NaN -> 0x7F
//   GEMM_Q_E2M1      OCP E2M1: round to nearest even, saturating at +-6
//                    (cvt.rn.satfinite.e2m1x2.f32); NaN -> 0x7; packed
//   GEMM_Q_MXFP4/8   OCP MX block scaling: per 32 consecutive elements of a
//                    row, X = floor(log2(amax)) - emax (2 for E2M1, 8 for
//                    E4M3) clamped to [-127, 127], UE8M0 code X + 127, and the
//                    elements quantised from v * 2^-X (exact scaling); an
//                    all-zero block gets code 0, a block holding NaN or Inf
//                    code 0xFF with zero elements
//
// One warp per 32-element MX block: the block maximum is one __reduce_max_sync
// over the magnitudes' bit patterns (non-negative floats order as integers).
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/mlpgemm.h"
#include "kernels.h"

namespace mlpg {

namespace {

// floatToE4M3, main.swift:6-27, on the f32 bit pattern.
__device__ __forceinline__ uint32_t q_e4m3_ref(float x) {
  if (isnan(x)) return 0x7F;
  const uint32_t sign = x < 0.f ? 0x80u : 0u;
  const float ax = fabsf(x);
  if (ax == 0.f) return sign;
  if (ax >= 448.f) return sign | 0x7E;
  const uint32_t bits = __float_as_uint(ax);
  int e = (int)((bits >> 23) & 0xFF) - 127 + 7;
  const uint32_t mant = bits & 0x7FFFFF;
  if (e <= 0) return sign;
  if (e >= 15) return sign | 0x7E;
  uint32_t m3 = (mant >> 20) + ((mant >> 19) & 1u);
  if (m3 == 8) {
    m3 = 0;
    e += 1;
    if (e >= 15) return sign | 0x7E;
  }
  return sign | ((uint32_t)e << 3) | m3;
}

__device__ __forceinline__ uint32_t q_e4m3_rne(float x) {
  if (isnan(x)) return 0x7F;
  unsigned short d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(0.f), "f"(x));
  return d & 0xFFu;
}

__device__ __forceinline__ uint32_t q_e2m1_rne(float x) {
  if (isnan(x)) x = 6.f;   // no NaN in E2M1: the positive maximum
  uint32_t d;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
      : "=r"(d)
      : "f"(0.f), "f"(x));
  return d & 0xFu;
}

template <int FMT>
__global__ void __launch_bounds__(256) quant_elem_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                                         long count) {
  // one pair of elements per thread and step (E2M1: one packed byte)
  const long pairs = (count + 1) / 2;
  for (long t = blockIdx.x * 256L + threadIdx.x; t < pairs; t += (long)gridDim.x * 256L) {
    const long i = 2 * t;
    const float a = src[i];
    const bool has_b = i + 1 < count;
    const float b = has_b ? src[i + 1] : 0.f;
    if constexpr (FMT == GEMM_Q_E2M1) {
      dst[t] = (uint8_t)(q_e2m1_rne(a) | (q_e2m1_rne(b) << 4));
    } else {
      const uint32_t qa = FMT == GEMM_Q_E4M3_REF ? q_e4m3_ref(a) : q_e4m3_rne(a);
      dst[i] = (uint8_t)qa;
      if (has_b) dst[i + 1] = (uint8_t)(FMT == GEMM_Q_E4M3_REF ? q_e4m3_ref(b) : q_e4m3_rne(b));
    }
  }
}

// floor(log2(a)) of a finite a > 0, subnormals included
__device__ __forceinline__ int floor_log2(uint32_t bits) {
  const int e = (int)(bits >> 23);
  if (e > 0) return e - 127;
  return (31 - __clz(bits & 0x7FFFFF)) - 149;   // subnormal: mantissa * 2^-149
}

// 2^p as a float for p in [-127, 127]
__device__ __forceinline__ float exp2_int(int p) {
  return p >= -126 ? __uint_as_float((uint32_t)(p + 127) << 23) : __uint_as_float(0x00400000u);
}

template <int ELEM>   // 0: E2M1 elements, 1: E4M3 elements
__global__ void __launch_bounds__(256) quant_mx_kernel(const float* __restrict__ src, uint8_t* __restrict__ vals,
                                                       uint8_t* __restrict__ scales, long rows, long cols) {
  const int lane = threadIdx.x & 31;
  const long nb = cols / 32;
  const long blk = blockIdx.x * 8L + (threadIdx.x >> 5);   // warp-uniform
  if (blk >= rows * nb) return;
  const long at = blk * 32 + lane;                         // = r * cols + b * 32 + lane
  const float v = src[at];
  const bool bad = __any_sync(0xffffffffu, !isfinite(v));
  const uint32_t amax = __reduce_max_sync(0xffffffffu, isfinite(v) ? (__float_as_uint(v) & 0x7FFFFFFFu) : 0u);
  constexpr int kEmax = ELEM == 0 ? 2 : 8;
  int X = 0;
  uint32_t code;
  if (bad) {
    code = 0xFF;
  } else if (amax == 0) {
    code = 0;
    X = -127;
  } else {
    X = floor_log2(amax) - kEmax;
    X = X < -127 ? -127 : (X > 127 ? 127 : X);
    code = (uint32_t)(X + 127);
  }
  uint32_t q = 0;
  if (!bad) {
    const float s = v * exp2_int(-X);   // exact: a power-of-two scaling
    q = ELEM == 0 ? q_e2m1_rne(s) : q_e4m3_rne(s);
  }
  if constexpr (ELEM == 0) {
    const uint32_t hi = __shfl_down_sync(0xffffffffu, q, 1);
    if ((lane & 1) == 0) vals[at / 2] = (uint8_t)(q | (hi << 4));
  } else {
    vals[at] = (uint8_t)q;
  }
  if (lane == 0) scales[blk] = (uint8_t)code;
}

}  // namespace

cudaError_t launch_quant(int format, const float* src, void* dst, void* scales, long rows, long cols,
                         int num_sms, cudaStream_t st) {
  const long count = rows * cols;
  uint8_t* d = static_cast<uint8_t*>(dst);
  const int sms = num_sms > 0 ? num_sms : 148;
  const long pairs = (count + 1) / 2;
  long g = (pairs + 255) / 256;
  if (g > 8L * sms) g = 8L * sms;
  switch (format) {
    case GEMM_Q_E4M3_REF: quant_elem_kernel<GEMM_Q_E4M3_REF><<<(unsigned)g, 256, 0, st>>>(src, d, count); break;
    case GEMM_Q_E4M3: quant_elem_kernel<GEMM_Q_E4M3><<<(unsigned)g, 256, 0, st>>>(src, d, count); break;
    case GEMM_Q_E2M1: quant_elem_kernel<GEMM_Q_E2M1><<<(unsigned)g, 256, 0, st>>>(src, d, count); break;
    case GEMM_Q_MXFP4:
    case GEMM_Q_MXFP8: {
      const long blocks = rows * (cols / 32);
      const unsigned grid = (unsigned)((blocks + 7) / 8);
      uint8_t* s = static_cast<uint8_t*>(scales);
      if (format == GEMM_Q_MXFP4) quant_mx_kernel<0><<<grid, 256, 0, st>>>(src, d, s, rows, cols);
      else quant_mx_kernel<1><<<grid, 256, 0, st>>>(src, d, s, rows, cols);
      break;
    }
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace mlpg
