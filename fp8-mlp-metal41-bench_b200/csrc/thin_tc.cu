// thin_tc.cu -- thin rows (N <= 16) on the tensor cores, weights as the A operand.
//
// The reference serves decode-shaped calls (N <= 16) with its 16x32 tile
// (main.swift:146-150) over the same matmul2d kernels (fp8_mlp.metal:60-276).
// Here the product is computed transposed, Y^T[M,N] = W^T[M,K] . X^T[K,N]:
// 128 weight rows (128 output columns of Y) fill the MMA's M = 128, and the
// <= 16 rows of X are its N = 16 (rows past N are zero-filled by TMA).  The
// weight stream -- the only large operand -- moves by TMA into a deep
// shared-memory ring, and the CUDA cores do no multiply-adds at all.
//
// Work is split stream-K: a unit is one K stage of one 128-row weight tile,
// the grid is one CTA per SM, and CTA c takes units [c*U/G, (c+1)*U/G), so
// every SM streams the same number of weight bytes.  A tile whose K range is
// shared by several CTAs is summed through the workspace: each contributor
// writes its 128 x 16 partial to slot (tile + c), and the last to arrive on
// the tile's counter (one per 32-row quadrant) adds the slots in CTA order, so
// the result does not depend on arrival order.
//
//   warp 0      TMA producer: weight stage (128 rows x 128 bytes) + X boxes
//   warp 1      TMEM allocator + single-thread MMA issuer (accumulators of
//               16 columns, double-buffered across the CTA's tile segments)
//   warps 4-7   epilogue: tcgen05.ld 32 rows x 16 columns per warp, then Y
//               (whole tile) or a partial slot (shared tile)
//   warps 8-15  converters (A16 kinds): raw weight stage -> f16 A sub-stages
//
// Kinds:
//   fp16        kind::f16, A = W^T MN-major (W [K,M] half), straight from TMA
//   i8i8        kind::i8 (S8 x S8 -> S32, exact), A MN-major
//   f8f8        kind::f8f6f4 (E4M3 x E4M3), A MN-major
//   int8, fp8   kind::f16 after exact widening of the [K,M] bytes to f16
//   mxfp4       kind::f16 after widening E2M1 * 2^(s-127-c) to f16 (K-major);
//               c is a per-row exponent offset chosen from the row's scales
//               in the CTA's K range, so that every block of the row is exact
//               in f16 down to 2^-24 of its largest block; the f32 partial is
//               multiplied back by 2^c (exact)
//
// Every wait is bounded (ptx.cuh); on expiry the kernel records an error word,
// lets its TMA copies land, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>
#include <type_traits>

#include "formats.cuh"
#include "kernels.h"
#include "partition.cuh"
#include "ptx.cuh"
#include "tmap.h"
#include "widen.cuh"

namespace mlpg {

namespace {

constexpr int kTBM = 128;          // weight rows per tile (MMA M)
constexpr int kTBN = 16;           // X rows per tile (MMA N)
constexpr int kTRow = 128;         // bytes per shared-memory row (one 128-byte swizzle row)
constexpr int kMaxThinCtas = 1024;  // partial slots reserved for CTAs
constexpr size_t kThinCounterBytes = 64 * 1024;
constexpr int kMaxThinTiles = (int)(kThinCounterBytes / (4 * sizeof(unsigned)));
constexpr int kConvWarps = 16;

enum ThinMode : int { kThinDirect = 0, kThinWidenKM = 1, kThinWidenMX = 2 };

template <int DT>
struct ThinT;
template <>
struct ThinT<kFP16> {
  static constexpr int mode = kThinDirect, kind = kKindF16, wbits = 16;
  static constexpr uint32_t fmt = 0, cfmt = 1;   // F16 x F16 -> F32
};
template <>
struct ThinT<kI8I8> {
  static constexpr int mode = kThinDirect, kind = kKindI8, wbits = 8;
  static constexpr uint32_t fmt = 1, cfmt = 2;   // S8 x S8 -> S32
};
template <>
struct ThinT<kF8F8> {
  static constexpr int mode = kThinDirect, kind = kKindF8F6F4, wbits = 8;
  static constexpr uint32_t fmt = 0, cfmt = 1;   // E4M3 x E4M3 -> F32
};
template <>
struct ThinT<kINT8> {
  static constexpr int mode = kThinWidenKM, kind = kKindF16, wbits = 8;
  static constexpr uint32_t fmt = 0, cfmt = 1;
};
template <>
struct ThinT<kFP8> {
  static constexpr int mode = kThinWidenKM, kind = kKindF16, wbits = 8;
  static constexpr uint32_t fmt = 0, cfmt = 1;
};
template <>
struct ThinT<kMXFP4> {
  static constexpr int mode = kThinWidenMX, kind = kKindF16, wbits = 4;
  static constexpr uint32_t fmt = 0, cfmt = 1;
};

template <int DT, int STAGES>
struct ThinCfg {
  using T = ThinT<DT>;
  static constexpr bool DIRECT = T::mode == kThinDirect;
  static constexpr bool MX = T::mode == kThinWidenMX;
  static constexpr int THREADS = DIRECT ? 256 : 256 + 32 * kConvWarps;
  // one unit = one raw weight stage of 128 rows x 128 bytes
  static constexpr int UNIT_K = kTRow * 8 / T::wbits;          // K elements: 64 / 128 / 256
  static constexpr int CV_K = 128;                              // K elements per converted f16 stage
  static constexpr int SUBS = DIRECT ? 1 : UNIT_K / CV_K;       // converted stages per unit (1 or 2)
  static constexpr int W_BYTES = kTBM * kTRow;                   // 16 KB
  static constexpr int X_BOX = kTBN * kTRow;                     // 16 rows x 128 bytes of K
  static constexpr int X_BOX_K = DIRECT && T::wbits == 8 ? 128 : 64;   // K elements per X box
  static constexpr int X_BOXES = UNIT_K / X_BOX_K;
  static constexpr int RAW_BYTES = W_BYTES + X_BOXES * X_BOX;    // 18 / 20 / 24 KB
  static constexpr int RAW_STAGES = STAGES;
  static constexpr int CV_STAGES = DIRECT ? 0 : 3;
  // mxfp4 rows are K-major, one row per converter thread: the widened rows go
  // straight to TMEM (the MMA's A operand may sit there), which keeps the
  // 4x-expanded f16 stream out of shared memory.  The [K,M] bytes need a
  // transpose to become TMEM rows, so int8 / fp8 widen into shared memory.
  static constexpr bool A_TMEM = MX;
  static constexpr int CV_A_BYTES = A_TMEM ? 0 : kTBM * CV_K * 2;   // 128 rows x 128 f16 of K
  // a converted slot holds its A tile (shared-memory kinds) and a copy of its
  // two X boxes, so that a raw slot is free again as soon as it is converted
  static constexpr int CV_SLOT = CV_A_BYTES + 2 * X_BOX;
  static constexpr int A_COL0 = 2 * kTBN;                        // TMEM: after the two accumulators
  static constexpr int A_COLS = CV_K / 2;                        // TMEM columns per converted stage
  static constexpr uint32_t TMEM_COLS = A_TMEM ? 256u : 32u;
  static constexpr int CV_OFF = RAW_STAGES * RAW_BYTES;
  static constexpr int OFFS_OFF = CV_OFF + CV_STAGES * CV_SLOT;   // mxfp4: 2 x 128 exponent offsets
  static constexpr int BAR_OFF = OFFS_OFF + (MX ? 2 * kTBM * 4 : 0);
  static constexpr int SMEM_BYTES = BAR_OFF + 512 + 1024;        // + barriers + alignment slack
  static constexpr int MMAS = DIRECT ? 4 : 8;                     // per (sub-)stage, 32 bytes of K each
  // A (weights): MN-major for the [K,M] layouts -- two 64-column halves
  // (8 KB apart from TMA, 16 KB apart when converted) for 16-bit elements,
  // one 128-column atom for 8-bit -- and K-major for the widened mxfp4 rows
  // (two 128-byte swizzle atoms of K, 16 KB apart).  Per-MMA step: K rows x
  // 128 B, or 32 B inside a K-major atom.
  static constexpr bool A_MN = !MX;
  static constexpr uint32_t A_LBO =
      MX ? 16u : (DIRECT ? (T::wbits == 8 ? (uint32_t)W_BYTES : 64u * kTRow) : (uint32_t)CV_K * kTRow);
  static constexpr uint32_t A_STEP = MX ? 32u : (DIRECT && T::wbits == 8 ? 32u : 16u) * kTRow;
  static constexpr int A_GRP = MX ? 4 : MMAS;                      // MMAs per K-major atom
  static constexpr uint32_t A_GRP_STRIDE = (uint32_t)kTBM * kTRow;
  static constexpr uint32_t IDESC = (T::cfmt << 4) | (T::fmt << 7) | (T::fmt << 10) |
                                    ((A_MN ? 1u : 0u) << 15) | ((uint32_t)(kTBN >> 3) << 17) |
                                    ((uint32_t)(kTBM >> 4) << 24);
  static_assert(RAW_BYTES % 1024 == 0 && CV_SLOT % 1024 == 0, "swizzle atoms need 1 KB alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(STAGES <= 10, "barrier array");
  static_assert(!A_TMEM || A_COL0 + CV_STAGES * A_COLS <= (int)TMEM_COLS, "TMEM budget");
};

// default ring depth: as deep as shared memory allows
template <int DT>
constexpr int thin_stages() {
  return ThinT<DT>::mode == kThinDirect ? 10 : (ThinT<DT>::mode == kThinWidenMX ? 8 : 5);
}

struct ThinBars {
  uint64_t raw_full[10];
  uint64_t raw_empty[10];
  uint64_t cv_full[4];
  uint64_t cv_empty[4];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t off_full[2];    // mxfp4: a segment's row offsets written
  uint64_t off_empty[2];   // mxfp4: ... and read by all their users
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(ThinBars) <= 512, "barrier area");

struct ThinParams {
  void* Y;
  const uint8_t* wscale;   // mxfp4: [M, K/32]
  void* part;              // partial slots: [(tiles + G)][4 quadrants][16 n][32 rows]
  unsigned* counters;      // [tiles][4 quadrants]
  int N, K, M;
  int tiles, upt, units;   // weight tiles, units per tile, all units
  int* dev_err;
};

// Exponent offset c that brings UE8M0 scales in [mn, mx] into the window
// where E2M1 * 2^(s-127-c) is an exact f16 (s - c in [104, 140]); when the
// range is wider than the window the largest blocks stay exact.
__device__ __forceinline__ int mx_offset(int mn, int mx) {
  if (mx > 140) return mx - 140;
  if (mn < 104) return max(mn - 104, mx - 140);
  return 0;
}

template <int DT, int STAGES>
__global__ void __launch_bounds__(ThinCfg<DT, STAGES>::THREADS, 1)
    tc_thin_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   ThinParams p) {
  using C = ThinCfg<DT, STAGES>;
  using T = typename C::T;
  using Acc = std::conditional_t<DT == kI8I8, int, float>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  ThinBars* bars = reinterpret_cast<ThinBars*>(smem + C::BAR_OFF);
  int* offs = reinterpret_cast<int*>(smem + C::OFFS_OFF);   // mxfp4: [2][128]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  AbortCtl ctl{p.dev_err, &bars->abort_flag};
  int u0, u1;
  cta_range(blockIdx.x, gridDim.x, p.units, u0, u1);
  const int tile0 = u0 / p.upt, ks0 = u0 - tile0 * p.upt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::RAW_STAGES; ++s) {
      mbar_init(&bars->raw_full[s], 1);
      // released by the MMAs (direct kinds) or by every converter warp
      mbar_init(&bars->raw_empty[s], C::DIRECT ? 1 : kConvWarps);
    }
    for (int s = 0; s < C::CV_STAGES; ++s) {
      mbar_init(&bars->cv_full[s], kConvWarps);
      mbar_init(&bars->cv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 4);
      mbar_init(&bars->off_full[b], 4);                   // converter warps 8-11 write
      mbar_init(&bars->off_empty[b], 4 + kConvWarps - 4);  // the epilogue and the other converters read
    }
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0 && lane == 0) {
    // ------------------------------ TMA producer ------------------------------
    uint32_t stage = 0, phase = 0;
    uint32_t filled_parity[C::RAW_STAGES];
    bool filled[C::RAW_STAGES];
    for (int s = 0; s < C::RAW_STAGES; ++s) filled[s] = false, filled_parity[s] = 0;
    bool ok = true;
    int tile = tile0, ks = ks0;
    for (int u = u0; u < u1; ++u) {
      if (!mbar_wait(&bars->raw_empty[stage], phase ^ 1u, ctl, 0x100 + stage)) { ok = false; break; }
      unsigned char* w_dst = smem + stage * C::RAW_BYTES;
      uint64_t* bar = &bars->raw_full[stage];
      mbar_arrive_expect_tx(bar, C::RAW_BYTES);
      // x coordinates: elements of the map; multiples of 64 halfs or 128 bytes
      if constexpr (C::MX) {
        tma_load_2d(w_dst, &tmW, bar, ks * kTRow, tile * kTBM);          // [M,K/2] bytes
      } else if constexpr (T::wbits == 16) {
        tma_load_2d(w_dst, &tmW, bar, tile * kTBM, ks * C::UNIT_K);      // [K,M] halfs: 64 columns
        tma_load_2d(w_dst + C::W_BYTES / 2, &tmW, bar, tile * kTBM + 64, ks * C::UNIT_K);
      } else {
        tma_load_2d(w_dst, &tmW, bar, tile * kTBM, ks * C::UNIT_K);      // [K,M] bytes: 128 columns
      }
#pragma unroll
      for (int b = 0; b < C::X_BOXES; ++b)
        tma_load_2d(w_dst + C::W_BYTES + b * C::X_BOX, &tmX, bar, ks * C::UNIT_K + b * C::X_BOX_K, 0);
      filled[stage] = true;
      filled_parity[stage] = phase;
      if (++stage == C::RAW_STAGES) { stage = 0; phase ^= 1u; }
      if (++ks == p.upt) { ks = 0; ++tile; }
    }
    if (!ok) {
      // let copies already in flight land before the CTA exits
      for (int s = 0; s < C::RAW_STAGES; ++s) {
        if (!filled[s]) continue;
        const uint32_t a = smem_u32(&bars->raw_full[s]);
        const unsigned long long t0 = global_ns();
        while (!mbar_try_wait(a, filled_parity[s]) && global_ns() - t0 < kWaitTimeoutNs) {}
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------ MMA issuer --------------------------------
    uint32_t rs = 0, rph = 0, cs = 0, cph = 0;
    int seg = 0, ks = ks0;
    bool ok = true;
    const uint32_t sbase = smem_u32(smem);
    for (int u = u0; u < u1 && ok; ++u) {
      const bool first = u == u0 || ks == 0;
      const bool last = u == u1 - 1 || ks == p.upt - 1;
      const int buf = seg & 1;
      if (first) {
        if (!mbar_wait(&bars->acc_empty[buf], ((uint32_t)(seg >> 1) & 1u) ^ 1u, ctl, 0x200 + buf)) break;
        tc_fence_after();
      }
      if constexpr (C::DIRECT) {
        // converted kinds read only converted slots (cv_full); their raw slots
        // are recycled by the converters and may run ahead of this thread
        if (!mbar_wait(&bars->raw_full[rs], rph, ctl, 0x300 + rs)) break;
        tc_fence_after();
      }
      const uint32_t d_tmem = tmem_base + (uint32_t)(buf * kTBN);
      const uint32_t w_addr = sbase + rs * C::RAW_BYTES;
#pragma unroll 1
      for (int sub = 0; sub < C::SUBS; ++sub) {
        uint32_t a_addr = w_addr, b_addr = w_addr + C::W_BYTES;
        if constexpr (!C::DIRECT) {
          if (!mbar_wait(&bars->cv_full[cs], cph, ctl, 0x500 + cs)) { ok = false; break; }
          tc_fence_after();
          a_addr = sbase + C::CV_OFF + cs * C::CV_SLOT;
          b_addr = a_addr + C::CV_A_BYTES;
        }
#pragma unroll
        for (int kk = 0; kk < C::MMAS; ++kk) {
          const uint64_t bd = sdesc_sw128(b_addr + (kk / 4) * C::X_BOX + (kk % 4) * 32, 16, 1024);
          const uint32_t acc = (first && sub == 0 && kk == 0) ? 0u : 1u;
          if constexpr (C::A_TMEM) {
            // K = 16 per MMA: 8 TMEM columns of the converted stage
            tc_mma_f16_ta(d_tmem, tmem_base + (uint32_t)(C::A_COL0 + cs * C::A_COLS + kk * 8), bd, C::IDESC, acc);
          } else {
            const uint64_t ad = sdesc_sw128(
                a_addr + (kk / C::A_GRP) * C::A_GRP_STRIDE + (kk % C::A_GRP) * C::A_STEP, C::A_LBO, 1024);
            tc_mma<T::kind>(d_tmem, ad, bd, C::IDESC, acc);
          }
        }
        if constexpr (!C::DIRECT) {
          tc_commit(&bars->cv_empty[cs]);
          if (++cs == C::CV_STAGES) { cs = 0; cph ^= 1u; }
        }
      }
      if (!ok) break;
      if constexpr (C::DIRECT) {
        tc_commit(&bars->raw_empty[rs]);
        if (++rs == C::RAW_STAGES) { rs = 0; rph ^= 1u; }
      }
      if (last) {
        tc_commit(&bars->acc_full[buf]);
        ++seg;
      }
      if (++ks == p.upt) ks = 0;
    }
  } else if (warp >= 8) {
    // ------------------------------ converters --------------------------------
    if constexpr (!C::DIRECT) {
      const int ct = threadIdx.x - 256;   // 0..511
      const int r = ct & 127;             // mxfp4: weight row of this thread
      const int bq = ct >> 7;             // mxfp4: which of a converted stage's four k-blocks
      const int kbpr = p.K / 32;
      uint32_t rs = 0, rph = 0, cs = 0, cph = 0;
      int seg = 0, tile = tile0, ks = ks0, c_row = 0;
      bool ok = true;
      int sc_next[2] = {127, 127};
      auto load_scales = [&](int t, int k, int (&dst)[2]) {
        const int mm = t * kTBM + r;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int kb = k * 8 + 4 * i + bq;
          dst[i] = (mm < p.M && kb < kbpr) ? (int)__ldg(p.wscale + (size_t)mm * kbpr + kb) : 127;
        }
      };
      for (int u = u0; u < u1 && ok; ++u) {
        const bool first = u == u0 || ks == 0;
        const bool last = u == u1 - 1 || ks == p.upt - 1;
        const int m = tile * kTBM + r;
        int sc[2] = {127, 127};
        if constexpr (C::MX) {
          const int buf = seg & 1;
          const uint32_t par = (uint32_t)(seg >> 1) & 1u;
          if (first) {
            if (ct < 128) {
              // the row's scales over this segment's K range -> offset c
              if (!mbar_wait_warp(&bars->off_empty[buf], par ^ 1u, ctl, 0x800 + buf)) break;
              const int kend = min(p.upt - 1, ks + (u1 - 1 - u));
              int mn = 255, mx = 0;
              if (m < p.M) {
                const int b1 = min(kbpr, (kend + 1) * 8);
                const uint8_t* sp = p.wscale + (size_t)m * kbpr;
                int b = ks * 8;
                if ((reinterpret_cast<uintptr_t>(sp + b) & 3u) == 0) {
                  uint32_t mn4 = 0xFFFFFFFFu, mx4 = 0u;   // per-byte minimum and maximum
                  for (; b + 4 <= b1; b += 4) {
                    const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(sp + b));
                    mn4 = __vminu4(mn4, w);
                    mx4 = __vmaxu4(mx4, w);
                  }
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    mn = min(mn, (int)((mn4 >> (8 * i)) & 0xFFu));
                    mx = max(mx, (int)((mx4 >> (8 * i)) & 0xFFu));
                  }
                }
                for (; b < b1; ++b) {
                  const int s = __ldg(sp + b);
                  mn = min(mn, s);
                  mx = max(mx, s);
                }
              }
              c_row = mx >= mn ? mx_offset(mn, mx) : 0;
              offs[buf * kTBM + r] = c_row;
              __syncwarp();
              if (lane == 0) mbar_arrive(&bars->off_full[buf]);
            } else {
              if (!mbar_wait_warp(&bars->off_full[buf], par, ctl, 0x900 + buf)) break;
              c_row = offs[buf * kTBM + r];
              __syncwarp();
              if (lane == 0) mbar_arrive(&bars->off_empty[buf]);
            }
          }
          // this thread's scale bytes (k-block 4*sub + bq) of this unit, loaded
          // one unit ahead so that their latency hides behind a unit's work
          if (u == u0) load_scales(tile, ks, sc_next);
#pragma unroll
          for (int i = 0; i < 2; ++i) sc[i] = sc_next[i];
          if (u + 1 < u1) {
            if (ks + 1 == p.upt) load_scales(tile + 1, 0, sc_next);
            else load_scales(tile, ks + 1, sc_next);
          }
        }
        if (!mbar_wait_warp(&bars->raw_full[rs], rph, ctl, 0x700 + rs)) break;
        const unsigned char* raw = smem + rs * C::RAW_BYTES;
#pragma unroll 1
        for (int sub = 0; sub < C::SUBS; ++sub) {
          if (!mbar_wait_warp(&bars->cv_empty[cs], cph ^ 1u, ctl, 0xA00 + cs)) { ok = false; break; }
          unsigned char* cv = smem + C::CV_OFF + cs * C::CV_SLOT;
          // this stage's two X boxes (4 KB, already in the MMA's layout): 8 bytes per thread
          *reinterpret_cast<uint2*>(cv + C::CV_A_BYTES + ct * 8) =
              *reinterpret_cast<const uint2*>(raw + C::W_BYTES + sub * 2 * C::X_BOX + ct * 8);
          if constexpr (C::MX) {
            // raw rows of 128 B (128-byte swizzle): k-block blk of row r is chunk
            // blk ^ (r & 7); its 32 E2M1 -> 16 TMEM columns (two f16 of K each) of
            // lane r, columns 16 * bq .. of the converted stage.  Warp w reaches
            // the TMEM lanes of quadrant w % 4, which holds rows r = 32 * (w % 4) + lane.
            const int blk = 4 * sub + bq;
            const uint4 w = *reinterpret_cast<const uint4*>(raw + r * kTRow + ((blk ^ (r & 7)) << 4));
            const uint32_t mul = f16x2_pow2(sc[sub] - 127 - c_row);
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
            uint32_t h[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint4 t = widen_e2m1x8(words[i], mul);
              h[4 * i] = t.x;
              h[4 * i + 1] = t.y;
              h[4 * i + 2] = t.z;
              h[4 * i + 3] = t.w;
            }
            tmem_st_32x32b_x16(tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) +
                                   (uint32_t)(C::A_COL0 + cs * C::A_COLS + 16 * bq),
                               h);
            tmem_st_wait();
          } else {
            // raw [128 K rows][128 B of M] -> two MN-major halves [128 K rows][64
            // columns of f16], 16 KB apart, 128-byte swizzle
#pragma unroll
            for (int it = 0; it < 4; ++it) {
              const int i = ct + 512 * it;
              const int c16 = i & 15, kr = i >> 4;
              const uint2 v = *reinterpret_cast<const uint2*>(raw + kr * kTRow + c16 * 8);
              const uint4 h = DT == kINT8 ? widen_i8x8(v) : widen_e4m3x8(v);
              const int j = c16 >> 3, c = c16 & 7;
              *reinterpret_cast<uint4*>(cv + j * (C::CV_K * kTRow) + kr * kTRow + ((c ^ (kr & 7)) << 4)) = h;
            }
          }
          fence_proxy_async_smem();   // generic-proxy writes -> visible to tcgen05.mma
          if constexpr (C::A_TMEM) tc_fence_before();   // tcgen05.st -> the MMA thread
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->cv_full[cs]);
          if (++cs == C::CV_STAGES) { cs = 0; cph ^= 1u; }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->raw_empty[rs]);
        if (++rs == C::RAW_STAGES) { rs = 0; rph ^= 1u; }
        if (last) ++seg;
        if (++ks == p.upt) { ks = 0; ++tile; }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------ epilogue ----------------------------------
    const int q = warp - 4;   // TMEM lane quadrant == warp % 4
    const int r = q * 32 + lane;
    const int G = gridDim.x;
    Acc* Y = reinterpret_cast<Acc*>(p.Y);
    Acc* part = reinterpret_cast<Acc*>(p.part);
    int seg = 0, tile = tile0, ks = ks0;
    for (int u = u0; u < u1; ++seg, ++tile) {
      const int n_units = min(p.upt - ks, u1 - u);
      const bool whole = ks == 0 && n_units == p.upt;
      const int buf = seg & 1;
      const uint32_t par = (uint32_t)(seg >> 1) & 1u;
      if (!mbar_wait_warp(&bars->acc_full[buf], par, ctl, 0x400 + buf)) break;
      tc_fence_after();
      uint32_t v[16];
      tmem_ld_32x32b_x16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kTBN), v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
      if constexpr (C::MX) {
        if (!mbar_wait_warp(&bars->off_full[buf], par, ctl, 0x600 + buf)) break;
        const int c = offs[buf * kTBM + r];
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->off_empty[buf]);
        if (c != 0) {
          const float f = __int_as_float((c + 127) << 23);   // 2^c, exact
#pragma unroll
          for (int n = 0; n < kTBN; ++n) v[n] = __float_as_uint(__uint_as_float(v[n]) * f);
        }
      }
      const int m = tile * kTBM + r;
      if (whole) {
        if (m < p.M)
          for (int n = 0; n < p.N; ++n) reinterpret_cast<uint32_t*>(Y)[(size_t)n * p.M + m] = v[n];
      } else {
        const int first = owner_of(tile * p.upt, G, p.units);
        const int lastc = owner_of(tile * p.upt + p.upt - 1, G, p.units);
        uint32_t* slot = reinterpret_cast<uint32_t*>(part) + ((size_t)(tile + blockIdx.x) * 4 + q) * (kTBN * 32);
#pragma unroll
        for (int n = 0; n < kTBN; ++n) slot[n * 32 + lane] = v[n];
        __threadfence();
        __syncwarp();
        unsigned* ctr = p.counters + tile * 4 + q;
        int is_last = 0;
        if (lane == 0) is_last = atomicAdd(ctr, 1u) == (unsigned)(lastc - first);
        is_last = __shfl_sync(0xffffffffu, is_last, 0);
        if (is_last) {
          __threadfence();
          // every contributor's 16 columns in flight at once, summed in CTA order
          Acc sum[kTBN];
#pragma unroll
          for (int n = 0; n < kTBN; ++n) sum[n] = 0;
          for (int cc = first; cc <= lastc; ++cc) {
            const Acc* src = part + ((size_t)(tile + cc) * 4 + q) * (kTBN * 32) + lane;
            Acc t[kTBN];
#pragma unroll
            for (int n = 0; n < kTBN; ++n) t[n] = __ldcg(src + n * 32);
#pragma unroll
            for (int n = 0; n < kTBN; ++n) sum[n] += t[n];
          }
          if (m < p.M) {
#pragma unroll
            for (int n = 0; n < kTBN; ++n)
              if (n < p.N) Y[(size_t)n * p.M + m] = sum[n];
          }
          if (lane == 0) *ctr = 0u;   // ready for the next launch
        }
      }
      u += n_units;
      ks = 0;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int DT, int STAGES = thin_stages<DT>()>
cudaError_t launch_thin_dt(const RunArgs& a, int grid_cap = 0) {
  using C = ThinCfg<DT, STAGES>;
  using T = typename C::T;
  CUtensorMap tmW, tmX;
  const CUtensorMapDataType u8 = CU_TENSOR_MAP_DATA_TYPE_UINT8, u16 = CU_TENSOR_MAP_DATA_TYPE_UINT16;
  bool ok;
  if constexpr (C::MX) {
    ok = make_map(&tmW, a.W, u8, (uint64_t)a.K / 2, (uint64_t)a.M, (uint64_t)a.K / 2, kTRow, kTBM);
  } else if constexpr (!C::DIRECT) {
    ok = make_map_plain(&tmW, a.W, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.M, kTBM, C::UNIT_K);
  } else if constexpr (T::wbits == 16) {
    ok = make_map(&tmW, a.W, u16, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.M * 2, 64, C::UNIT_K);
  } else {
    ok = make_map(&tmW, a.W, u8, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.M, kTBM, C::UNIT_K);
  }
  if (!ok) return cudaErrorInvalidValue;
  if constexpr (x_is_half(DT))
    ok = make_map(&tmX, a.X, u16, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K * 2, 64, kTBN);
  else
    ok = make_map(&tmX, a.X, u8, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, kTRow, kTBN);
  if (!ok) return cudaErrorInvalidValue;

  ThinParams p;
  p.Y = a.Y;
  p.wscale = a.wscale;
  p.counters = static_cast<unsigned*>(a.ws);
  p.part = static_cast<char*>(a.ws) + kThinCounterBytes;
  p.N = a.N;
  p.K = a.K;
  p.M = a.M;
  p.tiles = (a.M + kTBM - 1) / kTBM;
  p.upt = (a.K + C::UNIT_K - 1) / C::UNIT_K;
  p.units = p.tiles * p.upt;
  p.dev_err = a.dev_err;
  int grid = grid_cap > 0 ? grid_cap : a.num_sms;
  if (grid > kMaxThinCtas) grid = kMaxThinCtas;
  if (grid > p.units) grid = p.units;   // every CTA owns at least one unit
  auto k = tc_thin_kernel<DT, STAGES>;
  // per device: dynamic shared memory opt-in done (locked: host threads may
  // launch on one device at the same time)
  static std::mutex mu;
  static unsigned attr_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(attr_mask & (1u << (dev & 31)))) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
      if (e != cudaSuccess) return e;
      attr_mask |= 1u << (dev & 31);
    }
  }
  k<<<grid, C::THREADS, C::SMEM_BYTES, a.stream>>>(tmW, tmX, p);
  return cudaGetLastError();
}

}  // namespace

bool thin_supported(int dt, int N, int K, int M) {
  if (N < 1 || N > kTBN || K < 1 || M < 1) return false;
  if ((M + kTBM - 1) / kTBM > kMaxThinTiles) return false;
  switch (dt) {
    case kFP16: return M % 8 == 0 && K % 8 == 0;                      // 16-byte TMA strides
    case kINT8:
    case kFP8: return M % 16 == 0 && K % 8 == 0;
    case kI8I8:
    case kF8F8: return M % 16 == 0 && K % 16 == 0;
    case kMXFP4: return K % 32 == 0;
    default: return false;
  }
}

size_t thin_workspace(int dt, int N, int K, int M) {
  if (!thin_supported(dt, N, K, M)) return 0;
  const size_t tiles = (size_t)(M + kTBM - 1) / kTBM;
  return kThinCounterBytes + (tiles + kMaxThinCtas) * 4 * kTBN * 32 * 4;
}

cudaError_t launch_thin(const RunArgs& a) {
  if (!thin_supported(a.dt, a.N, a.K, a.M)) return cudaErrorInvalidValue;
  if (!a.ws || a.ws_bytes < thin_workspace(a.dt, a.N, a.K, a.M)) return cudaErrorInvalidValue;
  switch (a.dt) {
    case kFP16: return launch_thin_dt<kFP16>(a);
    case kI8I8: return launch_thin_dt<kI8I8>(a);
    case kF8F8: return launch_thin_dt<kF8F8>(a);
    case kINT8: return launch_thin_dt<kINT8>(a);
    case kFP8: return launch_thin_dt<kFP8>(a);
    case kMXFP4: return launch_thin_dt<kMXFP4>(a);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mlpg
