// gemv.cu -- CUDA-core split-K GEMM for thin rows (N <= 16, the decode row of
// the suite) and the any-shape fallback.
//
// The reference serves N = 1 with its smallest Metal tiles (defaultTile,
// main.swift:148-154: 16x32 for N <= 16).  Here thin rows get a kernel of
// their own: the weights are streamed from HBM once with 128-bit coalesced
// loads, decoded in registers, multiplied by activations held in shared
// memory (decoded to f32 once per CTA), reduced across warps in shared
// memory and across K-splits through a caller-provided workspace.  The last
// CTA of each output tile to finish sums the K-split partials in a fixed
// order, so results are deterministic (and exact for i8i8).
//
// Two weight layouts:
//   [K,M] "MN-major" (fp16, int8, i8i8, fp8, f8f8, f4f4): a thread owns a
//        16/8/4-byte run of one weight row (8..32 columns); the 8 warps of
//        a CTA walk interleaved K rows.
//   [M,K] "K-major" (the mxfp4 family): a warp owns 4 output columns; each
//        lane takes 16-byte blocks of 32 E2M1 values (one UE8M0 scale each)
//        and the warp reduces with shuffles.
#include <cuda_runtime.h>
#include <cstdint>
#include <type_traits>

#include "formats.cuh"
#include "kernels.h"

namespace mlpg {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

struct GemvParams {
  const void* X;
  const void* W;
  void* Y;
  const uint8_t* xscale;
  const uint8_t* wscale;
  int N, K, M;
  int ksplit;
  int kchunk;           // K elements per split (multiple of 32)
  void* part;           // [ksplit][N][M] partial sums (float, or int32 for i8i8)
  unsigned* counters;   // one per (row block, column block)
};

// Bytes per weight element, times two (FP4 packs two per byte).
template <int DT>
constexpr int w_bytes_x2() {
  return DT == kFP16 ? 4 : (DT == kF4F4 ? 1 : 2);
}

// ---- exact widening to f16 pairs, and f16 x f16 -> f32 multiply-adds ----------
// The products are formed by fma.rn.f32.f16 (f16 multiplicands, f32 addend):
// an f16 x f16 product has at most 22 significant bits, so it is exact in
// f32 and the accumulation is ordinary f32 -- no f16 rounding anywhere.

// int8 x4 -> two f16x2 (exact): bias to unsigned, place each byte under the
// exponent of 1024 (0x64xx = 1024 + byte), subtract 1152.
__device__ __forceinline__ void i8x4_to_h2(uint32_t v, uint32_t& lo, uint32_t& hi) {
  const uint32_t a = v ^ 0x80808080u;
  uint32_t t0 = __byte_perm(a, 0x64646464u, 0x4140), t1 = __byte_perm(a, 0x64646464u, 0x4342);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(t0), "r"(0x64806480u));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(t1), "r"(0x64806480u));
}

__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t two) {
  uint32_t d;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"((unsigned short)two));
  return d;
}

// 8 E2M1 (low nibble first) -> 4 f16x2
__device__ __forceinline__ void e2m1x8_to_h2(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// a0 += w.lo * x ; a1 += w.hi * x   (one activation, two weight columns)
__device__ __forceinline__ void fma2_bcast(float& a0, float& a1, uint32_t w2, unsigned short x) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
      "fma.rn.f32.f16 %0, l, %3, %0;\n\tfma.rn.f32.f16 %1, h, %3, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(w2), "h"(x));
}

// a += w.lo * x.lo + w.hi * x.hi   (two consecutive K elements)
__device__ __forceinline__ void fma2_dot(float& a, uint32_t w2, uint32_t x2) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\tmov.b32 {wl, wh}, %1;\n\tmov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.f16 %0, wl, xl, %0;\n\tfma.rn.f32.f16 %0, wh, xh, %0;\n\t}"
      : "+f"(a)
      : "r"(w2), "r"(x2));
}

// Widen one thread's weight chunk (LW bytes of one [K,M] row) to f16 pairs.
template <int DT, int LW>
__device__ __forceinline__ void widen_chunk(const uint32_t (&raw)[LW / 4],
                                            uint32_t (&h)[LW * 2 / w_bytes_x2<DT>() / 2]) {
#pragma unroll
  for (int i = 0; i < LW / 4; ++i) {
    if constexpr (DT == kFP16) {
      h[i] = raw[i];
    } else if constexpr (DT == kINT8) {
      i8x4_to_h2(raw[i], h[2 * i], h[2 * i + 1]);
    } else if constexpr (w_is_e4m3(DT)) {
      h[2 * i] = e4m3x2_to_h2(raw[i]);
      h[2 * i + 1] = e4m3x2_to_h2(raw[i] >> 16);
    } else {   // f4f4
      uint32_t q[4];
      e2m1x8_to_h2(raw[i], q);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[4 * i + j] = q[j];
    }
  }
}

// Element-wise guarded decode of weight (k, m) for the MN-major layouts.
template <int DT>
__device__ __forceinline__ float load_w_mn(const void* W, int k, int m, int M) {
  const size_t i = (size_t)k * M + m;
  if constexpr (DT == kFP16) return dec_f16(reinterpret_cast<const uint16_t*>(W)[i]);
  else if constexpr (w_is_i8(DT)) return (float)reinterpret_cast<const int8_t*>(W)[i];
  else if constexpr (w_is_e4m3(DT)) return dec_e4m3(reinterpret_cast<const uint8_t*>(W)[i]);
  else {
    const uint8_t b = reinterpret_cast<const uint8_t*>(W)[i >> 1];
    return dec_e2m1((i & 1) ? (b >> 4) : (b & 0xF));
  }
}

template <typename Acc>
__device__ __forceinline__ void finish_tile(const GemvParams& p, Acc* red, int n0, int NR,
                                            int m0, int CPC) {
  // red[NR][CPC] holds this CTA's (row block, column block, K split) result.
  const int tid = threadIdx.x;
  const int ks = blockIdx.y;
  Acc* Y = reinterpret_cast<Acc*>(p.Y);
  if (p.ksplit == 1) {
    for (int i = tid; i < NR * CPC; i += kThreads) {
      const int n = n0 + i / CPC, m = m0 + i % CPC;
      if (n < p.N && m < p.M) Y[(size_t)n * p.M + m] = red[i];
    }
    return;
  }
  Acc* part = reinterpret_cast<Acc*>(p.part);
  for (int i = tid; i < NR * CPC; i += kThreads) {
    const int n = n0 + i / CPC, m = m0 + i % CPC;
    if (n < p.N && m < p.M) part[((size_t)ks * p.N + n) * p.M + m] = red[i];
  }
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  const unsigned tile = blockIdx.z * gridDim.x + blockIdx.x;
  if (tid == 0) {
    const unsigned ticket = atomicAdd(&p.counters[tile], 1u);
    s_last = (ticket == (unsigned)p.ksplit - 1u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < NR * CPC; i += kThreads) {
    const int n = n0 + i / CPC, m = m0 + i % CPC;
    if (n < p.N && m < p.M) {
      Acc s = 0;
      for (int q = 0; q < p.ksplit; ++q) {  // fixed order: deterministic
        s += __ldcg(&part[((size_t)q * p.N + n) * p.M + m]);
      }
      Y[(size_t)n * p.M + m] = s;
    }
  }
  if (tid == 0) p.counters[tile] = 0u;  // ready for the next launch
}

// ---------------------------------------------------------------------------
// [K,M] weights
// ---------------------------------------------------------------------------
// A CTA owns a slab of CL x LW bytes of columns (CL lanes side by side on
// one row) and the K range of its split; its 256/CL row-lanes walk that
// range with stride 256/CL rows, 8 rows in flight per thread.  Activations
// sit in shared memory as f16 (exact for half, E4M3 and E2M1 inputs), or
// int8 for i8i8.  The row-lanes are reduced in shared memory in a fixed
// order, the K splits through the workspace (finish_tile).
template <int DT, int NR, int LW, int CL>
__global__ void __launch_bounds__(kThreads) gemv_mn_kernel(GemvParams p) {
  using Acc = std::conditional_t<DT == kI8I8, int, float>;
  constexpr int E = LW * 2 / w_bytes_x2<DT>();  // weights (columns) per thread
  constexpr int CPC = CL * E;                   // columns per CTA
  constexpr int H = E / 2;                      // f16 pairs per thread
  constexpr int RL = kThreads / CL;             // row-lanes
  constexpr int U = 8;                          // rows in flight per thread
  static_assert(DT != kI8I8 || U % 4 == 0, "dp4a takes groups of 4 rows");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int kc = p.kchunk;                      // multiple of 32
  unsigned char* xsb = smem_raw;                // [NR][kc] f16 (or int8)
  Acc* red = reinterpret_cast<Acc*>(smem_raw + (size_t)NR * kc * 2);   // [RL][NR][CPC]

  const int m0 = blockIdx.x * CPC;
  const int kb = blockIdx.y * kc;
  const int ke = min(p.K, kb + kc);
  const int n0 = blockIdx.z * NR;
  const int tid = threadIdx.x;
  const int cl = tid % CL, rl = tid / CL;

  for (int i = tid; i < NR * kc; i += kThreads) {
    const int n = i / kc, k = kb + i % kc;
    const bool in = n0 + n < p.N && k < ke;
    if constexpr (DT == kI8I8) {
      reinterpret_cast<int8_t*>(xsb)[i] = in ? reinterpret_cast<const int8_t*>(p.X)[(size_t)(n0 + n) * p.K + k] : 0;
    } else {
      reinterpret_cast<__half*>(xsb)[i] = __float2half_rn(in ? load_x<DT>(p.X, p.xscale, n0 + n, k, p.K) : 0.f);
    }
  }
  __syncthreads();

  Acc acc[NR][E];
#pragma unroll
  for (int n = 0; n < NR; ++n)
#pragma unroll
    for (int j = 0; j < E; ++j) acc[n][j] = 0;

  const int mc = m0 + cl * E;   // first column owned by this thread
  const size_t rb = (size_t)p.M * w_bytes_x2<DT>() / 2;   // bytes per weight row
  const bool vec = (mc + E <= p.M) && ((size_t)p.M * w_bytes_x2<DT>() % 2 == 0) && (rb % LW == 0);
  const uint8_t* wbase = reinterpret_cast<const uint8_t*>(p.W) + (size_t)mc * w_bytes_x2<DT>() / 2;

  if (vec) {
    // rows k = kb + U*rl*... : row-lane rl takes rows kb + U*rl + i (i < U), then jumps by U*RL
    for (int k0 = kb + U * rl; k0 < ke; k0 += U * RL) {
      uint32_t raw[U][LW / 4];
#pragma unroll
      for (int r = 0; r < U; ++r) {
        const int k = k0 + r;
        if (k < ke) {
          const uint8_t* src = wbase + (size_t)k * rb;
          if constexpr (LW == 16) {
            const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src));
            raw[r][0] = v.x; raw[r][1] = v.y; raw[r][2] = v.z; raw[r][3] = v.w;
          } else if constexpr (LW == 8) {
            const uint2 v = __ldcs(reinterpret_cast<const uint2*>(src));
            raw[r][0] = v.x; raw[r][1] = v.y;
          } else {
            raw[r][0] = __ldcs(reinterpret_cast<const unsigned int*>(src));
          }
        } else {
#pragma unroll
          for (int q = 0; q < LW / 4; ++q) raw[r][q] = 0;
        }
      }
      const int kl = k0 - kb;
      if constexpr (DT == kI8I8) {
        // 4x4 byte transposes, then dp4a over 4 K rows at a time
#pragma unroll
        for (int g = 0; g < U / 4; ++g) {
#pragma unroll
          for (int n = 0; n < NR; ++n) {
            const int x4 = *reinterpret_cast<const int*>(xsb + (size_t)n * kc + kl + 4 * g);
#pragma unroll
            for (int c = 0; c < LW / 4; ++c) {
              const uint32_t lo01 = __byte_perm(raw[4 * g][c], raw[4 * g + 1][c], 0x5140);
              const uint32_t hi01 = __byte_perm(raw[4 * g][c], raw[4 * g + 1][c], 0x7362);
              const uint32_t lo23 = __byte_perm(raw[4 * g + 2][c], raw[4 * g + 3][c], 0x5140);
              const uint32_t hi23 = __byte_perm(raw[4 * g + 2][c], raw[4 * g + 3][c], 0x7362);
              acc[n][4 * c + 0] = __dp4a((int)__byte_perm(lo01, lo23, 0x5410), x4, acc[n][4 * c + 0]);
              acc[n][4 * c + 1] = __dp4a((int)__byte_perm(lo01, lo23, 0x7632), x4, acc[n][4 * c + 1]);
              acc[n][4 * c + 2] = __dp4a((int)__byte_perm(hi01, hi23, 0x5410), x4, acc[n][4 * c + 2]);
              acc[n][4 * c + 3] = __dp4a((int)__byte_perm(hi01, hi23, 0x7632), x4, acc[n][4 * c + 3]);
            }
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < U; ++r) {
          uint32_t h[H];
          widen_chunk<DT, LW>(raw[r], h);
#pragma unroll
          for (int n = 0; n < NR; ++n) {
            const unsigned short xv = reinterpret_cast<const unsigned short*>(xsb)[(size_t)n * kc + kl + r];
#pragma unroll
            for (int j = 0; j < H; ++j) fma2_bcast(acc[n][2 * j], acc[n][2 * j + 1], h[j], xv);
          }
        }
      }
    }
  } else {
    for (int k = kb + rl; k < ke; k += RL) {
      const int kl = k - kb;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        const int m = mc + j;
        if (m >= p.M) break;
        if constexpr (DT == kI8I8) {
          const int wv = reinterpret_cast<const int8_t*>(p.W)[(size_t)k * p.M + m];
#pragma unroll
          for (int n = 0; n < NR; ++n) acc[n][j] += (int)reinterpret_cast<const int8_t*>(xsb)[(size_t)n * kc + kl] * wv;
        } else {
          const float wv = load_w_mn<DT>(p.W, k, m, p.M);
#pragma unroll
          for (int n = 0; n < NR; ++n)
            acc[n][j] = fmaf(__half2float(reinterpret_cast<const __half*>(xsb)[(size_t)n * kc + kl]), wv, acc[n][j]);
        }
      }
    }
  }

  // row-lane reduction in a fixed order: red[rl][n][col], then column sums
#pragma unroll
  for (int n = 0; n < NR; ++n)
#pragma unroll
    for (int j = 0; j < E; ++j) red[((size_t)rl * NR + n) * CPC + cl * E + j] = acc[n][j];
  __syncthreads();
  Acc* out = red;   // the sums overwrite row-lane 0's slice, which thread t reads first
  for (int i = tid; i < NR * CPC; i += kThreads) {
    Acc sum = 0;
    for (int q = 0; q < RL; ++q) sum += red[(size_t)q * NR * CPC + i];
    out[i] = sum;   // only row-lane 0's entry i is overwritten, after it was read
  }
  __syncthreads();
  finish_tile<Acc>(p, out, n0, NR, m0, CPC);
}

// ---------------------------------------------------------------------------
// [M,K] weights (mxfp4 family): E2M1 packed along K, UE8M0 [M, K/32]
// ---------------------------------------------------------------------------
// Each 16-byte load is one 32-element block with one W scale (and, for
// mxfp4/a4 and mxfp4/a8, one X scale per row): the block's dot product of
// the unscaled f16 values is formed exactly in f32 and then multiplied by
// 2^(sw-127) * 2^(sx-127).
template <int DT, int NR>
__global__ void __launch_bounds__(kThreads) gemv_km_kernel(GemvParams p) {
  constexpr int RPW = 4;              // output columns per warp
  constexpr int CPC = kWarps * RPW;   // 32 columns per CTA
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int kc = p.kchunk;            // multiple of 32
  __half* xs = reinterpret_cast<__half*>(smem_raw);                       // [NR][kc] unscaled
  float* xsc = reinterpret_cast<float*>(smem_raw + (size_t)NR * kc * 2);   // [NR][kc/32]
  float* red = xsc + NR * (kc / 32);                                       // [NR][CPC]

  const int m0 = blockIdx.x * CPC;
  const int kb = blockIdx.y * kc;
  const int ke = min(p.K, kb + kc);
  const int n0 = blockIdx.z * NR;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kbpr = p.K / 32;

  for (int i = tid; i < NR * kc; i += kThreads) {
    const int n = i / kc, k = kb + i % kc;
    float v = 0.f;
    if (n0 + n < p.N && k < ke) {
      const size_t xi = (size_t)(n0 + n) * p.K + k;
      if constexpr (x_is_half(DT)) {
        v = dec_f16(reinterpret_cast<const uint16_t*>(p.X)[xi]);
      } else if constexpr (x_is_e4m3(DT)) {
        v = dec_e4m3(reinterpret_cast<const uint8_t*>(p.X)[xi]);
      } else {
        const uint8_t byte = reinterpret_cast<const uint8_t*>(p.X)[xi >> 1];
        v = dec_e2m1((xi & 1) ? (byte >> 4) : (byte & 0xF));
      }
    }
    xs[i] = __float2half_rn(v);   // exact: half, E4M3 and E2M1 values are f16 values
  }
  for (int i = tid; i < NR * (kc / 32); i += kThreads) {
    const int n = i / (kc / 32), blk = kb / 32 + i % (kc / 32);
    float sc = 1.f;
    if constexpr (x_scaled(DT)) {
      if (n0 + n < p.N && blk < kbpr) sc = dec_ue8m0(p.xscale[(size_t)(n0 + n) * kbpr + blk]);
    }
    xsc[i] = sc;
  }
  __syncthreads();

  float acc[NR][RPW];
#pragma unroll
  for (int n = 0; n < NR; ++n)
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[n][r] = 0.f;

  const int kblocks = (ke - kb) / 32;  // kchunk and K are multiples of 32
  const uint8_t* W = reinterpret_cast<const uint8_t*>(p.W);
  constexpr int BPL = 4;               // blocks per lane in flight, per row
  for (int b0 = lane; b0 < kblocks; b0 += 32 * BPL) {
    uint4 wv[BPL][RPW];
    float sc[BPL][RPW];
#pragma unroll
    for (int t = 0; t < BPL; ++t) {
      const int blk = b0 + 32 * t;
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int m = m0 + warp * RPW + r;
        if (m < p.M && blk < kblocks) {
          const int k = kb + blk * 32;
          wv[t][r] = __ldcs(reinterpret_cast<const uint4*>(W + ((size_t)m * p.K + k) / 2));
          sc[t][r] = dec_ue8m0(__ldg(p.wscale + (size_t)m * kbpr + k / 32));
        } else {
          wv[t][r] = make_uint4(0, 0, 0, 0);
          sc[t][r] = 0.f;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < BPL; ++t) {
      const int blk = b0 + 32 * t;
      if (blk >= kblocks) break;
#pragma unroll
      for (int n = 0; n < NR; ++n) {
        const uint4* xq = reinterpret_cast<const uint4*>(xs + (size_t)n * kc + blk * 32);
        uint32_t x2[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v = xq[q];
          x2[4 * q] = v.x; x2[4 * q + 1] = v.y; x2[4 * q + 2] = v.z; x2[4 * q + 3] = v.w;
        }
        const float xsn = xsc[n * (kc / 32) + blk];
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          float d = 0.f;
          const uint32_t words[4] = {wv[t][r].x, wv[t][r].y, wv[t][r].z, wv[t][r].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t h[4];
            e2m1x8_to_h2(words[q], h);
#pragma unroll
            for (int j = 0; j < 4; ++j) fma2_dot(d, h[j], x2[4 * q + j]);
          }
          acc[n][r] = fmaf(d, sc[t][r] * xsn, acc[n][r]);
        }
      }
    }
  }
  // butterfly reduction across lanes (same order on every run)
#pragma unroll
  for (int n = 0; n < NR; ++n)
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      float v = acc[n][r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[n][r] = v;
    }
  if (lane == 0) {
#pragma unroll
    for (int n = 0; n < NR; ++n)
#pragma unroll
      for (int r = 0; r < RPW; ++r) red[n * CPC + warp * RPW + r] = acc[n][r];
  }
  __syncthreads();
  finish_tile<float>(p, red, n0, NR, m0, CPC);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int DT>
constexpr bool is_kmajor() { return w_is_mx(DT); }

// Rows per CTA: 1, 2, 4 or 8 (larger N uses several row blocks).
inline int pick_nr(int N) { return N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : 8; }

// Lanes side by side on one weight row ([K,M] kernel): a narrow slab gives
// enough CTAs without splitting K; wide slabs for many rows (N > 1 runs are
// compute-heavier and prefer fewer, wider CTAs).
constexpr int kLanesPerRow = 4;

// Bytes loaded per thread per weight row, so that NR * E <= 64 accumulators.
template <int DT>
constexpr int pick_lw(int NR) {
  constexpr int bx2 = w_bytes_x2<DT>();
  int lw = 16;
  while (lw > 4 && NR * (lw * 2 / bx2) > 64) lw /= 2;
  return lw;
}

int cols_per_cta(int dt, int N) {
  if (dt == kMXFP4 || dt == kMX4X4 || dt == kMX8X4 || dt == kF8X4) return 32;
  const int nr = pick_nr(N);
  const int bx2 = dt == kFP16 ? 4 : (dt == kF4F4 ? 1 : 2);
  int lw = 16;
  while (lw > 4 && nr * (lw * 2 / bx2) > 64) lw /= 2;
  return kLanesPerRow * (lw * 2 / bx2);
}

// Workspace layout: [kCounterBytes of tile counters][ksplit * N * M partials].
// The counters sit at a fixed offset so that calls of different shapes that
// share one workspace never read another call's partial sums as counters.
constexpr size_t kCounterBytes = 64 * 1024;
constexpr int kMaxCounterTiles = (int)(kCounterBytes / sizeof(unsigned));

int kchunk_for(int K, int ksplit) {
  int kc = (K + ksplit - 1) / ksplit;
  return (kc + 31) / 32 * 32;
}

template <int DT, int NR>
cudaError_t launch_nr(const GemvParams& p, dim3 grid, cudaStream_t st) {
  size_t smem;
  if constexpr (is_kmajor<DT>()) {
    smem = (size_t)NR * p.kchunk * 2 + (size_t)NR * (p.kchunk / 32) * 4 + (size_t)NR * 32 * 4;
    auto k = gemv_km_kernel<DT, NR>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, st>>>(p);
  } else {
    constexpr int LW = pick_lw<DT>(NR);
    constexpr int E = LW * 2 / w_bytes_x2<DT>();
    constexpr int CL = kLanesPerRow;
    smem = (size_t)NR * p.kchunk * 2 + (size_t)(kThreads / CL) * NR * CL * E * 4;
    auto k = gemv_mn_kernel<DT, NR, LW, CL>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, st>>>(p);
  }
  return cudaGetLastError();
}

template <int DT>
cudaError_t launch_dt(const GemvParams& p, dim3 grid, int nr, cudaStream_t st) {
  switch (nr) {
    case 1: return launch_nr<DT, 1>(p, grid, st);
    case 2: return launch_nr<DT, 2>(p, grid, st);
    case 4: return launch_nr<DT, 4>(p, grid, st);
    default: return launch_nr<DT, 8>(p, grid, st);
  }
}

}  // namespace

__global__ void __launch_bounds__(512) l2_flush_kernel(const uint4* __restrict__ buf, size_t n16,
                                                       unsigned* __restrict__ never) {
  uint32_t x = 0;
  for (size_t i = blockIdx.x * 512ull + threadIdx.x; i < n16; i += (size_t)gridDim.x * 512ull) {
    const uint4 v = __ldcg(buf + i);
    x ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (x == 0x9E3779B9u && never) *never = x;   // keeps the loads; never taken for a zero buffer
}

cudaError_t launch_l2_flush(const void* buf, size_t bytes, int num_sms, cudaStream_t st) {
  l2_flush_kernel<<<4 * num_sms, 512, 0, st>>>(static_cast<const uint4*>(buf), bytes / 16, nullptr);
  return cudaGetLastError();
}

int gemv_auto_ksplit(int dt, int N, int K, int M, int num_sms) {
  const int nr = pick_nr(N);
  const long ctas = (long)((M + cols_per_cta(dt, N) - 1) / cols_per_cta(dt, N)) *
                    ((N + nr - 1) / nr);
  const long target = 4L * (num_sms > 0 ? num_sms : 148);
  int s = 1;
  if (ctas > kMaxCounterTiles) return 1;
  while (s < 64 && ctas * s < target && K / (2 * s) >= 64) s *= 2;
  return s;
}

size_t gemv_workspace(int dt, int ksplit, int N, int K, int M) {
  (void)dt;
  if (ksplit <= 1) return 0;
  const int kc = kchunk_for(K, ksplit);
  const int eff = (K + kc - 1) / kc;
  if (eff <= 1) return 0;
  return kCounterBytes + (size_t)eff * N * M * 4;
}

cudaError_t launch_gemv(const RunArgs& a, int ksplit) {
  if (ksplit < 1) ksplit = 1;
  GemvParams p;
  p.X = a.X;
  p.W = a.W;
  p.Y = a.Y;
  p.xscale = a.xscale;
  p.wscale = a.wscale;
  p.N = a.N;
  p.K = a.K;
  p.M = a.M;
  p.kchunk = kchunk_for(a.K, ksplit);
  p.ksplit = (a.K + p.kchunk - 1) / p.kchunk;
  const int nr = pick_nr(a.N);
  const int cpc = cols_per_cta(a.dt, a.N);
  dim3 grid((a.M + cpc - 1) / cpc, p.ksplit, (a.N + nr - 1) / nr);
  if (p.ksplit > 1) {
    if ((size_t)grid.x * grid.z > (size_t)kMaxCounterTiles) return cudaErrorInvalidValue;
    if (a.ws == nullptr || a.ws_bytes < gemv_workspace(a.dt, ksplit, a.N, a.K, a.M))
      return cudaErrorInvalidValue;
    p.counters = reinterpret_cast<unsigned*>(a.ws);
    p.part = reinterpret_cast<char*>(a.ws) + kCounterBytes;
  } else {
    p.part = nullptr;
    p.counters = nullptr;
  }
  switch (a.dt) {
    case kFP16: return launch_dt<kFP16>(p, grid, nr, a.stream);
    case kINT8: return launch_dt<kINT8>(p, grid, nr, a.stream);
    case kI8I8: return launch_dt<kI8I8>(p, grid, nr, a.stream);
    case kFP8: return launch_dt<kFP8>(p, grid, nr, a.stream);
    case kF8F8: return launch_dt<kF8F8>(p, grid, nr, a.stream);
    case kF4F4: return launch_dt<kF4F4>(p, grid, nr, a.stream);
    case kMXFP4: return launch_dt<kMXFP4>(p, grid, nr, a.stream);
    case kMX4X4: return launch_dt<kMX4X4>(p, grid, nr, a.stream);
    case kMX8X4: return launch_dt<kMX8X4>(p, grid, nr, a.stream);
    case kF8X4: return launch_dt<kF8X4>(p, grid, nr, a.stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mlpg
