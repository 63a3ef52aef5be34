// gemv_stream.cu -- persistent TMA-streaming GEMM for thin rows (N <= 16).
//
// The thin row of the suite (N = 1, K = 4096, M = 11008; main.swift:156-160)
// reads every weight byte once and does ~1 FLOP per byte: it is bound by HBM
// bandwidth, and what matters is keeping enough bytes in flight on every SM
// all the time.  Here one CTA runs per SM for the whole kernel:
//
//   warp 8        TMA producer: walks the CTA's share of the weights as 2-D
//                 boxes into a STAGES-deep shared-memory ring (no swizzle),
//                 completion on "full" mbarriers; for the [M,K] mxfp4
//                 weights it also brings the matching UE8M0 scale box
//   warps 0-7     consumers: widen the weights exactly to f16 pairs and
//                 multiply-add them with the f16 activations held in shared
//                 memory into f32 (fma.rn.f32.f16; dp4a for i8i8)
//
// Work split (stream-K): the weights are cut into units -- one box of
// RB rows of one column slab ([K,M] weights) or one K chunk of one group of
// 32 output rows ([M,K] weights) -- and every CTA takes a contiguous,
// equal run of units.  A run crosses slab boundaries freely; each (slab,
// CTA) piece is reduced inside the CTA in a fixed order and written as a
// partial sum, and the last CTA to finish a slab adds its partials in CTA
// order (deterministic, exact for int32).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <mutex>
#include <type_traits>

#include "formats.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace mlpg {

namespace {

constexpr int kSConsumers = 256;          // 8 consumer warps
constexpr int kSThreads = kSConsumers + 32;
constexpr int kStages = 8;
constexpr size_t kSCounterBytes = 64 * 1024;   // slab counters at offset 0 of the workspace
constexpr int kMaxStreamCtas = 1024;            // grid bound (one CTA per SM)

struct StreamParams {
  const void* X;
  const uint8_t* xscale;
  void* Y;
  const uint8_t* wscale;
  int N, K, M;
  int nslabs;          // column slabs ([K,M]) or 32-row groups ([M,K])
  int units_per_slab;  // boxes along K per slab
  int total_units;
  int nrowblk;         // row blocks of NR rows (gridDim.y)
  unsigned* counters;  // [nrowblk][nslabs]
  void* part;          // partial sums: [nrowblk][nslabs + gridDim.x][NR][slab columns]
  int* dev_err;
};

// contiguous unit range of CTA c
__device__ __forceinline__ void cta_range(int c, int G, int U, int& u0, int& u1) {
  u0 = (int)((long long)c * U / G);
  u1 = (int)((long long)(c + 1) * U / G);
}

// first CTA whose range contains unit u
__device__ __forceinline__ int owner_of(int u, int G, int U) {
  // largest c with c*U/G <= u
  int c = (int)(((long long)u * G + G - 1) / U);
  while (c > 0 && (long long)c * U / G > u) --c;
  while ((long long)(c + 1) * U / G <= u) ++c;
  return c;
}

// ---- exact widening helpers (as in gemv.cu) -------------------------------------
__device__ __forceinline__ void s_i8x4_to_h2(uint32_t v, uint32_t& lo, uint32_t& hi) {
  const uint32_t a = v ^ 0x80808080u;
  const uint32_t t0 = __byte_perm(a, 0x64646464u, 0x4140), t1 = __byte_perm(a, 0x64646464u, 0x4342);
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(t0), "r"(0x64806480u));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(t1), "r"(0x64806480u));
}
__device__ __forceinline__ uint32_t s_e4m3x2(uint32_t two) {
  uint32_t d;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"((unsigned short)two));
  return d;
}
__device__ __forceinline__ void s_e2m1x8(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}
__device__ __forceinline__ void s_fma2_bcast(float& a0, float& a1, uint32_t w2, unsigned short x) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
      "fma.rn.f32.f16 %0, l, %3, %0;\n\tfma.rn.f32.f16 %1, h, %3, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(w2), "h"(x));
}
__device__ __forceinline__ void s_fma2_dot(float& a, uint32_t w2, uint32_t x2) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\tmov.b32 {wl, wh}, %1;\n\tmov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.f16 %0, wl, xl, %0;\n\tfma.rn.f32.f16 %0, wh, xh, %0;\n\t}"
      : "+f"(a)
      : "r"(w2), "r"(x2));
}

template <int DT>
constexpr int s_wbytes_x2() {
  return DT == kFP16 ? 4 : (DT == kF4F4 ? 1 : 2);
}

// ---- layout configuration -----------------------------------------------------------
// [K,M] weights: slab = SB bytes of a row (64 B), box = SB x RB rows.
// [M,K] weights: slab = 32 output rows, box = 256 B (512 E2M1) x 32 rows,
//                plus a 16-byte x 32-row box of UE8M0 scales.
template <int DT, int NR>
struct SCfg {
  static constexpr bool KM = w_is_mx(DT);
  static constexpr int SB = 64;                              // [K,M]: slab bytes per row
  static constexpr int RB = 128;                             // [K,M]: rows per box
  static constexpr int SLAB_COLS = KM ? 32 : SB * 2 / s_wbytes_x2<DT>();
  static constexpr int BOX_BYTES = KM ? 256 * 32 : SB * RB;  // 8 KB
  static constexpr int SC_BYTES = KM ? 16 * 32 : 0;          // scale box (512 B)
  static constexpr int STAGE_BYTES = BOX_BYTES + SC_BYTES;
  static constexpr int K_PER_UNIT = KM ? 512 : RB;           // K elements per unit
  static constexpr int CL = SB / 16;                          // [K,M]: 16-byte lanes per row
  static constexpr int RL = kSConsumers / CL;                 // [K,M]: row-lanes (64)
  using Acc = std::conditional_t<DT == kI8I8, int, float>;
  static constexpr int E = KM ? 1 : 16 * 2 / s_wbytes_x2<DT>();   // accumulators per row of X
};

template <int DT, int NR>
__global__ void __launch_bounds__(kSThreads, 1)
    gemv_stream_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                       StreamParams p) {
  using C = SCfg<DT, NR>;
  using Acc = typename C::Acc;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* ring = smem_raw;                                      // kStages x STAGE_BYTES
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * C::STAGE_BYTES);
  uint64_t* empty = full + kStages;
  int* abort_flag = reinterpret_cast<int*>(empty + kStages);
  int* s_last = abort_flag + 1;
  // activations of this row block: [NR][K] f16 (or int8), X scales [NR][K/32]
  unsigned char* xsb = reinterpret_cast<unsigned char*>(abort_flag + 4);
  xsb = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(xsb) + 15) & ~uintptr_t(15));
  float* xsc = reinterpret_cast<float*>(xsb + (size_t)NR * p.K * 2);
  Acc* red = reinterpret_cast<Acc*>(xsc + (C::KM ? NR * (p.K / 32) : 0));   // reduction scratch

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int n0 = blockIdx.y * NR;
  AbortCtl ctl{p.dev_err, abort_flag};
  int u0, u1;
  cta_range(c, G, p.total_units, u0, u1);

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSConsumers / 32);   // one arrival per consumer warp
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  // activations for rows n0..n0+NR-1, all of K (exact in f16 / int8)
  for (int i = tid; i < NR * p.K; i += kSThreads) {
    const int n = i / p.K, k = i % p.K;
    const bool in = n0 + n < p.N;
    if constexpr (DT == kI8I8) {
      reinterpret_cast<int8_t*>(xsb)[i] = in ? reinterpret_cast<const int8_t*>(p.X)[(size_t)(n0 + n) * p.K + k] : 0;
    } else {
      float v = 0.f;
      if (in) {
        const size_t xi = (size_t)(n0 + n) * p.K + k;
        if constexpr (x_is_half(DT)) v = dec_f16(reinterpret_cast<const uint16_t*>(p.X)[xi]);
        else if constexpr (x_is_e4m3(DT)) v = dec_e4m3(reinterpret_cast<const uint8_t*>(p.X)[xi]);
        else {
          const uint8_t b = reinterpret_cast<const uint8_t*>(p.X)[xi >> 1];
          v = dec_e2m1((xi & 1) ? (b >> 4) : (b & 0xF));
        }
      }
      reinterpret_cast<__half*>(xsb)[i] = __float2half_rn(v);
    }
  }
  if constexpr (C::KM) {
    const int kb = p.K / 32;
    for (int i = tid; i < NR * kb; i += kSThreads) {
      const int n = i / kb, b = i % kb;
      float sc = 1.f;
      if constexpr (x_scaled(DT)) {
        if (n0 + n < p.N) sc = dec_ue8m0(p.xscale[(size_t)(n0 + n) * kb + b]);
      }
      xsc[i] = sc;
    }
  }
  __syncthreads();

  if (warp == kSConsumers / 32) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      for (int u = u0; u < u1; ++u) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, ctl, 0x910 + stage)) break;
        const int slab = u / p.units_per_slab, ku = u % p.units_per_slab;
        unsigned char* dst = ring + stage * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
        if constexpr (C::KM) {
          tma_load_2d(dst, &tmW, &full[stage], ku * 256, slab * 32);                 // bytes of K, rows
          tma_load_2d(dst + C::BOX_BYTES, &tmS, &full[stage], ku * 16, slab * 32);   // scale bytes, rows
        } else {
          tma_load_2d(dst, &tmW, &full[stage], slab * C::SB, ku * C::RB);            // bytes of M, rows of K
        }
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
    }
  } else {
    // ------------------------------ consumers ---------------------------------
    uint32_t stage = 0, phase = 0;
    bool dead = false;   // a bounded wait expired: keep walking units and barriers, skip work
    int u = u0;
    while (u < u1) {
      const int slab = u / p.units_per_slab;
      const int send = min(u1, (slab + 1) * p.units_per_slab);   // end of this slab in our run
      Acc acc[NR][C::E];
#pragma unroll
      for (int n = 0; n < NR; ++n)
#pragma unroll
        for (int j = 0; j < C::E; ++j) acc[n][j] = 0;
      for (; u < send; ++u) {
        const int ku = u % p.units_per_slab;
        if (!dead) {
          const bool got = mbar_wait(&full[stage], phase, ctl, 0x920 + stage);
          dead = !__all_sync(0xffffffffu, got);
        }
        const unsigned char* box = ring + stage * C::STAGE_BYTES;
        if (dead) {
          // no data: fall through to the barriers of this slab with zero sums
        } else if constexpr (!C::KM) {
          // thread (cl, rl): 16 bytes of rows rl and rl + RL of the box
          const int cl = tid % C::CL, rl = tid / C::CL;
          constexpr int E = 16 * 2 / s_wbytes_x2<DT>();   // columns per 16 bytes
#pragma unroll
          for (int rr = 0; rr < C::RB / C::RL; ++rr) {
            const int r = rl + rr * C::RL;
            const uint4 v = *reinterpret_cast<const uint4*>(box + r * C::SB + cl * 16);
            const int k = ku * C::RB + r;
            const uint32_t raw[4] = {v.x, v.y, v.z, v.w};
            if constexpr (DT == kI8I8) {
#pragma unroll
              for (int n = 0; n < NR; ++n) {
                const int xv = reinterpret_cast<const int8_t*>(xsb)[(size_t)n * p.K + k];
#pragma unroll
                for (int q = 0; q < 4; ++q)
#pragma unroll
                  for (int b = 0; b < 4; ++b) acc[n][4 * q + b] += xv * (int)(int8_t)(raw[q] >> (8 * b));
              }
            } else {
              uint32_t h[E / 2];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                if constexpr (DT == kFP16) h[q] = raw[q];
                else if constexpr (DT == kINT8) s_i8x4_to_h2(raw[q], h[2 * q], h[2 * q + 1]);
                else if constexpr (w_is_e4m3(DT)) { h[2 * q] = s_e4m3x2(raw[q]); h[2 * q + 1] = s_e4m3x2(raw[q] >> 16); }
                else { uint32_t t4[4]; s_e2m1x8(raw[q], t4);
#pragma unroll
                       for (int j = 0; j < 4; ++j) h[4 * q + j] = t4[j]; }
              }
#pragma unroll
              for (int n = 0; n < NR; ++n) {
                const unsigned short xv = reinterpret_cast<const unsigned short*>(xsb)[(size_t)n * p.K + k];
#pragma unroll
                for (int j = 0; j < E / 2; ++j) s_fma2_bcast(acc[n][2 * j], acc[n][2 * j + 1], h[j], xv);
              }
            }
          }
        } else {
          // thread t: row t/8 of the 32-row group, blocks (t%8) and (t%8)+8 of the 16 in the box
          const int r = tid >> 3, bsel = tid & 7;
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int blk = bsel + 8 * h2;
            const uint4 v = *reinterpret_cast<const uint4*>(box + r * 256 + blk * 16);
            const float ws = dec_ue8m0(box[C::BOX_BYTES + r * 16 + blk]);
            const int kblk = ku * 16 + blk;
            const uint32_t words[4] = {v.x, v.y, v.z, v.w};
            uint32_t h[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t t4[4];
              s_e2m1x8(words[q], t4);
#pragma unroll
              for (int j = 0; j < 4; ++j) h[4 * q + j] = t4[j];
            }
#pragma unroll
            for (int n = 0; n < NR; ++n) {
              const uint4* xq = reinterpret_cast<const uint4*>(xsb + ((size_t)n * p.K + kblk * 32) * 2);
              float d = 0.f;
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint4 xv = xq[q];
                s_fma2_dot(d, h[4 * q + 0], xv.x);
                s_fma2_dot(d, h[4 * q + 1], xv.y);
                s_fma2_dot(d, h[4 * q + 2], xv.z);
                s_fma2_dot(d, h[4 * q + 3], xv.w);
              }
              acc[n][0] = fmaf(d, ws * xsc[n * (p.K / 32) + kblk], acc[n][0]);
            }
          }
        }
        __syncwarp();
        if (lane == 0 && !dead) mbar_arrive(&empty[stage]);
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
      // ---- reduce this (slab, CTA) piece inside the CTA, in a fixed order ----
      Acc* out;
      if constexpr (!C::KM) {
        const int cl = tid % C::CL, rl = tid / C::CL;
        constexpr int E = 16 * 2 / s_wbytes_x2<DT>();
        // red[rl][n][col]
#pragma unroll
        for (int n = 0; n < NR; ++n)
#pragma unroll
          for (int j = 0; j < E; ++j) red[((size_t)rl * NR + n) * C::SLAB_COLS + cl * E + j] = acc[n][j];
        asm volatile("bar.sync 1, %0;" ::"n"(kSConsumers));
        for (int i = tid; i < NR * C::SLAB_COLS; i += kSConsumers) {
          Acc sum = 0;
          for (int q = 0; q < C::RL; ++q) sum += red[(size_t)q * NR * C::SLAB_COLS + i];
          red[i] = sum;
        }
        out = red;
      } else {
        // 8 threads per row: shuffle-reduce, then red[n][row]
#pragma unroll
        for (int n = 0; n < NR; ++n) {
          float v = acc[n][0];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          if ((tid & 7) == 0) red[n * 32 + (tid >> 3)] = v;
        }
        out = red;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kSConsumers));
      // ---- write the partial, and let the last contributor finish the slab ----
      const int first = owner_of(slab * p.units_per_slab, G, p.total_units);
      const int last = owner_of((slab + 1) * p.units_per_slab - 1, G, p.total_units);
      const int ncontrib = last - first + 1;
      Acc* part = reinterpret_cast<Acc*>(p.part) +
                  ((size_t)blockIdx.y * (p.nslabs + G) + (size_t)(slab + c)) * NR * C::SLAB_COLS;
      // slot (slab + c) is unique per (slab, contributor): contributors of a slab are consecutive CTAs
      for (int i = tid; i < NR * C::SLAB_COLS; i += kSConsumers) part[i] = out[i];
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kSConsumers));
      if (tid == 0) {
        const unsigned t = atomicAdd(&p.counters[blockIdx.y * p.nslabs + slab], 1u);
        *s_last = (t == (unsigned)ncontrib - 1u);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kSConsumers));
      if (*s_last) {
        __threadfence();
        Acc* Y = reinterpret_cast<Acc*>(p.Y);
        const Acc* base = reinterpret_cast<const Acc*>(p.part) + (size_t)blockIdx.y * (p.nslabs + G) * NR * C::SLAB_COLS;
        for (int i = tid; i < NR * C::SLAB_COLS; i += kSConsumers) {
          const int n = i / C::SLAB_COLS, col = i % C::SLAB_COLS;
          const int m = slab * C::SLAB_COLS + col;
          if (n0 + n >= p.N || m >= p.M) continue;
          Acc sum = 0;
          for (int q = first; q <= last; ++q)   // CTA order: deterministic
            sum += __ldcg(base + (size_t)(slab + q) * NR * C::SLAB_COLS + i);
          Y[(size_t)(n0 + n) * p.M + m] = sum;
        }
        if (tid == 0) p.counters[blockIdx.y * p.nslabs + slab] = 0u;   // ready for the next launch
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kSConsumers));
    }
  }
  __syncthreads();
}

// ---- host side ------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn s_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

bool s_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
           uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = s_encode();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int s_pick_nr(int N) { return N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : 8; }

struct SGeom {
  int nslabs, ups, units, slab_cols, nrowblk;
  size_t smem;
};

SGeom s_geom(int dt, int N, int K, int M) {
  SGeom g;
  const int nr = s_pick_nr(N);
  const bool km = w_is_mx(dt);
  const int bx2 = dt == kFP16 ? 4 : (dt == kF4F4 ? 1 : 2);
  g.slab_cols = km ? 32 : 64 * 2 / bx2;
  g.nslabs = (M + g.slab_cols - 1) / g.slab_cols;
  g.ups = km ? (K + 511) / 512 : (K + 127) / 128;
  g.units = g.nslabs * g.ups;
  g.nrowblk = (N + nr - 1) / nr;
  const size_t stage = km ? 256 * 32 + 512 : 64 * 128;
  const size_t red = km ? (size_t)nr * 32 * 4 : (size_t)64 * nr * g.slab_cols * 4;
  g.smem = kStages * stage + 2 * kStages * 8 + 64 + (size_t)nr * K * 2 + (km ? (size_t)nr * (K / 32) * 4 : 0) +
           red + 16;
  return g;
}

template <int DT, int NR>
cudaError_t s_launch(const RunArgs& a, int grid, const SGeom& g) {
  using C = SCfg<DT, NR>;
  CUtensorMap tmW, tmS;
  bool ok;
  if constexpr (C::KM) {
    ok = s_map(&tmW, a.W, (uint64_t)a.K / 2, (uint64_t)a.M, (uint64_t)a.K / 2, 256, 32) &&
         s_map(&tmS, a.wscale, (uint64_t)a.K / 32, (uint64_t)a.M, (uint64_t)a.K / 32, 16, 32);
  } else {
    const uint64_t rb = (uint64_t)a.M * s_wbytes_x2<DT>() / 2;
    ok = s_map(&tmW, a.W, rb, (uint64_t)a.K, rb, C::SB, C::RB);
    tmS = tmW;
  }
  if (!ok) return cudaErrorInvalidValue;
  StreamParams p;
  p.X = a.X;
  p.xscale = a.xscale;
  p.Y = a.Y;
  p.wscale = a.wscale;
  p.N = a.N;
  p.K = a.K;
  p.M = a.M;
  p.nslabs = g.nslabs;
  p.units_per_slab = g.ups;
  p.total_units = g.units;
  p.nrowblk = g.nrowblk;
  p.counters = static_cast<unsigned*>(a.ws);
  p.part = static_cast<char*>(a.ws) + kSCounterBytes;
  p.dev_err = a.dev_err;
  auto k = gemv_stream_kernel<DT, NR>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
  if (e != cudaSuccess) return e;
  k<<<dim3(grid, g.nrowblk), kSThreads, g.smem, a.stream>>>(tmW, tmS, p);
  return cudaGetLastError();
}

template <int DT>
cudaError_t s_launch_dt(const RunArgs& a, int grid, const SGeom& g) {
  switch (s_pick_nr(a.N)) {
    case 1: return s_launch<DT, 1>(a, grid, g);
    case 2: return s_launch<DT, 2>(a, grid, g);
    case 4: return s_launch<DT, 4>(a, grid, g);
    default: return s_launch<DT, 8>(a, grid, g);
  }
}

int s_grid(const SGeom& g, int num_sms) {
  return g.units < num_sms ? g.units : num_sms;
}

}  // namespace

bool stream_supported(int dt, int N, int K, int M) {
  if (N < 1 || N > 16 || K < 1 || M < 1) return false;
  {
    const int bx2 = dt == kFP16 ? 4 : (dt == kF4F4 ? 1 : 2);
    const int e = w_is_mx(dt) ? 1 : 32 / bx2;
    if (s_pick_nr(N) * e > 64) return false;   // accumulators per thread
  }
  if (w_is_mx(dt)) return K % 512 == 0 && (K / 32) % 16 == 0;
  const int bx2 = dt == kFP16 ? 4 : (dt == kF4F4 ? 1 : 2);
  const long rb2 = (long)M * bx2;   // 2 x row bytes
  if (rb2 % 2) return false;
  if ((rb2 / 2) % 16) return false;   // TMA row stride
  if (K % 128) return false;          // whole boxes along K
  // activations of one row block live in shared memory
  return s_geom(dt, N, K, M).smem <= 200 * 1024;
}

size_t stream_workspace(int dt, int N, int K, int M) {
  const SGeom g = s_geom(dt, N, K, M);
  const int nr = s_pick_nr(N);
  // one slot per (slab, contributing CTA); the grid is at most kMaxStreamCtas
  const size_t slots = (size_t)g.nrowblk * (g.nslabs + kMaxStreamCtas);
  return kSCounterBytes + slots * nr * g.slab_cols * 4;
}

cudaError_t launch_stream(const RunArgs& a) {
  if (!stream_supported(a.dt, a.N, a.K, a.M)) return cudaErrorInvalidValue;
  const SGeom g = s_geom(a.dt, a.N, a.K, a.M);
  if ((size_t)g.nrowblk * g.nslabs * sizeof(unsigned) > kSCounterBytes) return cudaErrorInvalidValue;
  if (!a.ws || a.ws_bytes < stream_workspace(a.dt, a.N, a.K, a.M)) return cudaErrorInvalidValue;
  const int grid = s_grid(g, a.num_sms < kMaxStreamCtas ? a.num_sms : kMaxStreamCtas);
  switch (a.dt) {
    case kFP16: return s_launch_dt<kFP16>(a, grid, g);
    case kINT8: return s_launch_dt<kINT8>(a, grid, g);
    case kI8I8: return s_launch_dt<kI8I8>(a, grid, g);
    case kFP8: return s_launch_dt<kFP8>(a, grid, g);
    case kF8F8: return s_launch_dt<kF8F8>(a, grid, g);
    case kF4F4: return s_launch_dt<kF4F4>(a, grid, g);
    case kMXFP4: return s_launch_dt<kMXFP4>(a, grid, g);
    case kMX4X4: return s_launch_dt<kMX4X4>(a, grid, g);
    case kMX8X4: return s_launch_dt<kMX8X4>(a, grid, g);
    case kF8X4: return s_launch_dt<kF8X4>(a, grid, g);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mlpg
