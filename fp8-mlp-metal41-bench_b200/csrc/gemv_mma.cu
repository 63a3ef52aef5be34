// gemv_mma.cu -- thin rows (N <= 16) on the warp-level tensor-core MMA.
//
// The reference serves decode-shaped calls (N <= 16) with its thin tile
// (main.swift:146-150) over the dtype kernels of fp8_mlp.metal (fp16 :60-125,
// int8 W8A16 :127-138, fp8 W8A16 :153-164, f8f8 :166-177, mxfp4 :199-276 and
// the block-scaled MX kinds :278-444).  At N <= 16 the weight stream is the
// whole cost.  This kernel reads every weight byte from HBM once, widens it
// exactly to f16 and multiplies it on the tensor cores with
// mma.sync.m16n8k16 (f16 x f16 -> f32): the weights are the A operand (16
// output columns per MMA), up to 8 rows of X the B operand.  Against the
// CUDA-core GEMV this drops the per-element multiply-add and its f16 -> f32
// unpacking; what remains per weight element is the widening (1/2 instruction
// for E4M3 and E2M1, 1.5 for int8, 1/2 for the k-pair shuffle of f16).
//
// Memory: each warp streams its weights through a ring of kStages shared-memory
// stages filled by cp.async (16-byte copies, zero-filled past the matrix), so
// kStages - 1 steps per warp -- about 128 KB per SM -- are in flight without
// holding registers; cp.async.wait_group is the only wait (no spin loops).
//
// Operand placement (MMA fragment layouts of m16n8k16; lane = 4 g + t):
//   A (16 x 16, row-major): lane holds rows g and g+8, K slots {2t, 2t+1} and
//   {2t+8, 2t+9};  B (16 x 8): K slots {2t, 2t+1}, {2t+8, 2t+9} of column g;
//   C (16 x 8, f32): rows g, g+8 of columns 2t, 2t+1.
// Rows of A and K slots may be assigned to weights freely, as long as B uses
// the same K assignment:
//   [K,M] weights (fp16, int8, fp8, f8f8): a warp owns a slab of 128 bytes of
//     every weight row; a step is 16 rows.  Lane (g, t) copies and reads the 16
//     bytes at 16 g of weight rows k0 + 4t + r (r = 0..3 -> slots 2t, 2t+1,
//     2t+8, 2t+9) and the 4 values x[k0 + 4t ..] of X row g.  MMA block b puts
//     output column CPT*g + 2b on A row g and CPT*g + 2b + 1 on row g+8 (CPT =
//     the lane's 16 or 8 columns), so an A register is one byte_perm of two
//     rows' words (plus the widening).  Every lane reads only what it copied.
//   [M,K] MX weights (E2M1, one UE8M0 scale per 32 along K): a warp owns 16
//     weight rows; a step is 4 blocks (128 K, 64 bytes per row).  In block b
//     lane (g, t) takes the 4 bytes at 4t of rows g and g+8, and the block's
//     two MMAs take k = 8t..8t+3 and 8t+4..8t+7: every MMA lies inside one
//     block, so the block's product lands in a fresh f32 tile that is folded
//     into the accumulator times 2^(s_w - 127) (and the X block scale of the
//     a4/a8 kinds) -- no f16 range limit on the scales.
//
// Work split (stream-K): a unit is one step of a group of 8 slabs (a CTA's 8
// warps, one slab each: 1 KB of every weight row for [K,M], 128 weight rows
// for [M,K]).  The persistent grid's CTAs take equal contiguous runs of units,
// group-major, so every SM streams the same number of bytes and the 8 warps
// of a CTA stay on the same K rows.  At each group boundary the CTA writes its
// tile straight to Y (group held by this CTA alone) or to a partial slot; the
// last CTA to arrive on a shared group adds the slots in CTA order, so the
// result does not depend on timing.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "formats.cuh"
#include "kernels.h"
#include "widen.cuh"

namespace mlpg {

namespace {

constexpr int kMThreads = 256;
constexpr int kMWarps = kMThreads / 32;
constexpr int kMCtasPerSm = 2;
constexpr int kMaxMCtas = 1024;               // partial slots reserved per row block
constexpr size_t kMCounterBytes = 64 * 1024;
constexpr size_t kMaxMSmem = 200 * 1024;
constexpr int kStages = 5;                    // cp.async ring depth per warp

struct MmaParams {
  const void* X;
  const void* W;
  void* Y;
  const uint8_t* xscale;
  const uint8_t* wscale;
  int N, K, M;
  int ngroups;          // groups of 8 slabs
  int ks;               // steps per group (along K)
  int units;            // ngroups * ks
  float* part;          // [row block][ngroups + kMaxMCtas][8 warps][NR][SW] partial slots
  unsigned* counters;   // [row block][ngroups] arrival counters (zero between launches)
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

// Stream-K partition (partition.cuh) in 32-bit arithmetic: the host keeps
// (units + 1) * grid below 2^32.
__device__ __forceinline__ void run_of(unsigned c, unsigned G, unsigned U, int& u0, int& u1) {
  u0 = (int)(c * U / G);
  u1 = (int)((c + 1) * U / G);
}
__device__ __forceinline__ int owner32(unsigned u, unsigned G, unsigned U) {
  unsigned c = (u * G + G - 1) / U;   // largest c with c*U/G <= u, up to rounding
  while (c > 0 && c * U / G > u) --c;
  while ((c + 1) * U / G <= u) ++c;
  return (int)c;
}

// next (group, step) in group-major order
__device__ __forceinline__ void next_unit(int& grp, int& j, int ks) {
  if (++j == ks) {
    j = 0;
    ++grp;
  }
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two int8 (bytes 0, 1 or 2, 3 of p, already biased by 0x80) -> f16x2, exact:
// each byte under the exponent of 1024, minus 1152 (= 1024 + 128).
__device__ __forceinline__ uint32_t i8pair_lo(uint32_t p) {
  return hsub2_u32(__byte_perm(p, 0x64646464u, 0x4140), 0x64806480u);
}
__device__ __forceinline__ uint32_t i8pair_hi(uint32_t p) {
  return hsub2_u32(__byte_perm(p, 0x64646464u, 0x4342), 0x64806480u);
}

// f16 pair of the byte pair (bytes 0, 1) / (bytes 2, 3) of p, exact.
template <int DT>
__device__ __forceinline__ uint32_t pair_lo(uint32_t p) {
  if constexpr (w_is_i8(DT)) return i8pair_lo(p);
  else return cvt_e4m3x2(p);
}
template <int DT>
__device__ __forceinline__ uint32_t pair_hi(uint32_t p) {
  if constexpr (w_is_i8(DT)) return i8pair_hi(p);
  else return cvt_e4m3x2(p >> 16);
}

// The CTA's tile of one group, acc in the C layout, goes to Y (the group is
// held by this CTA alone) or to the CTA's partial slot; the last CTA to arrive
// on a shared group adds the slots in CTA order.  col(b, h) maps C rows (g for
// h = 0, g+8 for h = 1) of MMA block b to the warp's output columns.  Every
// thread of the CTA calls this at the same unit.
template <int NR, int SW, int NB, typename ColFn>
__device__ __forceinline__ void finish_group(const MmaParams& p, float (&acc)[NB][4], int grp, int n0,
                                             ColFn col) {
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = lane & 3;
  const int G = gridDim.x, c = blockIdx.x;
  const int first = owner32(grp * p.ks, G, p.units), last = owner32((grp + 1) * p.ks - 1, G, p.units);
  float* Y = static_cast<float*>(p.Y);
  const int m0 = (grp * kMWarps + warp) * SW;   // first output column of this warp's slab
  constexpr int TILE = kMWarps * NR * SW;        // floats of one CTA's group tile
  float* slots = p.part + (size_t)blockIdx.z * (p.ngroups + kMaxMCtas) * TILE;
  float* mine = slots + (size_t)(grp + c) * TILE + (size_t)warp * NR * SW;
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int n = 2 * t + (q & 1), ci = col(b, q >> 1);
      if (n < NR) {
        if (first == last) {
          if (n0 + n < p.N && m0 + ci < p.M) Y[(size_t)(n0 + n) * p.M + m0 + ci] = acc[b][q];
        } else {
          mine[n * SW + ci] = acc[b][q];
        }
      }
      acc[b][q] = 0.f;
    }
  if (first == last) return;
  __threadfence();
  __syncthreads();
  unsigned* ctr = p.counters + (size_t)blockIdx.z * p.ngroups + grp;
  if (tid == 0) s_last = atomicAdd(ctr, 1u) == (unsigned)(last - first);
  __syncthreads();
  if (s_last) {
    __threadfence();
    // element i = tid + 256 j of the tile; the slots of 4 contributors x JT
    // elements are loaded together, then added in CTA order
    constexpr int J = (TILE + kMThreads - 1) / kMThreads, JT = J < 8 ? J : 8;
    for (int j0 = 0; j0 < J; j0 += JT) {
      float v[JT];
#pragma unroll
      for (int jj = 0; jj < JT; ++jj) v[jj] = 0.f;
      for (int q0 = first; q0 <= last; q0 += 4) {
        float a[4][JT];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq)
#pragma unroll
          for (int jj = 0; jj < JT; ++jj) {
            const int i = tid + (j0 + jj) * kMThreads;
            a[qq][jj] = (q0 + qq <= last && i < TILE) ? __ldcg(slots + (size_t)(grp + q0 + qq) * TILE + i) : 0.f;
          }
#pragma unroll
        for (int qq = 0; qq < 4; ++qq)
#pragma unroll
          for (int jj = 0; jj < JT; ++jj)
            if (q0 + qq <= last) v[jj] += a[qq][jj];
      }
#pragma unroll
      for (int jj = 0; jj < JT; ++jj) {
        const int i = tid + (j0 + jj) * kMThreads;
        const int w = i / (NR * SW), n = (i / SW) % NR, ci = i % SW;
        const int m = (grp * kMWarps + w) * SW + ci;
        if (i < TILE && n0 + n < p.N && m < p.M) Y[(size_t)(n0 + n) * p.M + m] = v[jj];
      }
    }
    if (tid == 0) *ctr = 0u;   // ready for the next launch
  }
  __syncthreads();   // s_last is read before the next group reuses it
}

// ---------------------------------------------------------------------------
// [K,M] weights: fp16, int8 (W8A16), fp8 (W8A16), f8f8
// ---------------------------------------------------------------------------
template <int DT>
struct MnT {
  static constexpr int EB = DT == kFP16 ? 2 : 1;        // bytes per weight element
  static constexpr int SW = 128 / EB;                   // output columns per slab (128 bytes of a row)
  static constexpr int NB = SW / 16;                    // MMA blocks per warp
  static constexpr int CPT = SW / 8;                    // contiguous columns per lane
  static constexpr int X_OFF = 4 * 32 * 16;             // W: [4 rows per lane][32 lanes][16 B]
  static constexpr int STAGE = X_OFF + 32 * 8;          // + X fragments [32 lanes][8 B]
};

template <int DT, int NR>
__global__ void __launch_bounds__(kMThreads, kMCtasPerSm) gemv_mma_mn_kernel(MmaParams p) {
  using T = MnT<DT>;
  constexpr int SW = T::SW, NB = T::NB, CPT = T::CPT, STAGE = T::STAGE;
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.z * NR;
  int u0, u1;
  run_of(blockIdx.x, gridDim.x, p.units, u0, u1);
  if (u0 >= u1) return;   // CTA-uniform

  const uint32_t ring = (uint32_t)__cvta_generic_to_shared(smem) + (uint32_t)(warp * kStages * STAGE);
  const size_t rowb = (size_t)p.M * T::EB;
  const uint8_t* W = static_cast<const uint8_t*>(p.W);
  constexpr int XB = x_is_half(DT) ? 2 : 1;   // bytes per X element
  const bool xrow = g < NR && n0 + g < p.N;
  const uint8_t* xr = static_cast<const uint8_t*>(p.X) + (size_t)(xrow ? n0 + g : 0) * p.K * XB;

  // unit u: group u / ks, K rows 16 (u % ks) ..; this warp's slab is group * 8 + warp
  auto issue = [&](int grp, int j, int stage) {
    const uint32_t st = ring + (uint32_t)(stage * STAGE);
    const int k0 = 16 * j + 4 * t;
    const size_t colb = (size_t)(grp * kMWarps + warp) * 128 + 16 * g;
    const bool colok = colb < rowb;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int k = k0 + r;
      const bool ok = colok && k < p.K;
      cp_async16(st + (uint32_t)((r * 32 + lane) * 16), ok ? W + (size_t)k * rowb + colb : W, ok ? 16u : 0u);
    }
    const bool xok = xrow && k0 < p.K;
    const uint8_t* xs = xok ? xr + (size_t)k0 * XB : xr;
    if constexpr (XB == 2) cp_async8(st + T::X_OFF + lane * 8, xs, xok ? 8u : 0u);
    else cp_async4(st + T::X_OFF + lane * 8, xs, xok ? 4u : 0u);
  };

  float acc[NB][4];
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[b][q] = 0.f;

  auto compute = [&](int stage) {
    const uint32_t st = ring + (uint32_t)(stage * STAGE);
    uint32_t b0, b1;
    if constexpr (XB == 2) {
      const uint2 xv = lds64(st + T::X_OFF + lane * 8);
      b0 = xv.x;
      b1 = xv.y;
    } else {
      const uint32_t xv = lds32(st + T::X_OFF + lane * 8);
      b0 = cvt_e4m3x2(xv);
      b1 = cvt_e4m3x2(xv >> 16);
    }
    uint4 wv[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) wv[r] = lds128(st + (uint32_t)((r * 32 + lane) * 16));
    const uint32_t w[4][4] = {{wv[0].x, wv[0].y, wv[0].z, wv[0].w},
                              {wv[1].x, wv[1].y, wv[1].z, wv[1].w},
                              {wv[2].x, wv[2].y, wv[2].z, wv[2].w},
                              {wv[3].x, wv[3].y, wv[3].z, wv[3].w}};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (T::EB == 2) {
        // word j of a row holds columns 2j, 2j+1: MMA block j
        mma_f16(acc[j], __byte_perm(w[0][j], w[1][j], 0x5410), __byte_perm(w[0][j], w[1][j], 0x7632),
                __byte_perm(w[2][j], w[3][j], 0x5410), __byte_perm(w[2][j], w[3][j], 0x7632), b0, b1);
      } else {
        // word j holds columns 4j..4j+3: MMA blocks 2j (4j, 4j+1) and 2j+1 (4j+2, 4j+3)
        uint32_t r0 = w[0][j], r1 = w[1][j], r2 = w[2][j], r3 = w[3][j];
        if constexpr (w_is_i8(DT)) {
          r0 ^= 0x80808080u;
          r1 ^= 0x80808080u;
          r2 ^= 0x80808080u;
          r3 ^= 0x80808080u;
        }
        const uint32_t lo01 = __byte_perm(r0, r1, 0x5140), hi01 = __byte_perm(r0, r1, 0x7362);
        const uint32_t lo23 = __byte_perm(r2, r3, 0x5140), hi23 = __byte_perm(r2, r3, 0x7362);
        mma_f16(acc[2 * j], pair_lo<DT>(lo01), pair_hi<DT>(lo01), pair_lo<DT>(lo23), pair_hi<DT>(lo23), b0, b1);
        mma_f16(acc[2 * j + 1], pair_lo<DT>(hi01), pair_hi<DT>(hi01), pair_lo<DT>(hi23), pair_hi<DT>(hi23), b0,
                b1);
      }
    }
  };
  // C row g of block b is column CPT*g + 2b of the slab, row g+8 the next one
  auto col = [&](int b, int h) { return CPT * g + 2 * b + h; };

  int igrp = u0 / p.ks, ij = u0 - igrp * p.ks;   // next unit to copy
  int grp = igrp, cgrp = igrp, cj = ij;            // group in acc; unit to multiply
#pragma unroll
  for (int q = 0; q < kStages - 1; ++q) {
    if (u0 + q < u1) {
      issue(igrp, ij, q);
      next_unit(igrp, ij, p.ks);
    }
    cp_async_commit();
  }
  int stage = 0;
  for (int u = u0; u < u1; ++u) {
    cp_async_wait<kStages - 2>();   // this lane's copies of unit u have landed
    // refill the stage read in the previous step: this lane has consumed it,
    // and no other lane reads it
    if (u + kStages - 1 < u1) {
      issue(igrp, ij, stage == 0 ? kStages - 1 : stage - 1);
      next_unit(igrp, ij, p.ks);
    }
    cp_async_commit();
    if (cgrp != grp) {
      finish_group<NR, SW, NB>(p, acc, grp, n0, col);
      grp = cgrp;
    }
    compute(stage);
    next_unit(cgrp, cj, p.ks);
    stage = stage == kStages - 1 ? 0 : stage + 1;
  }
  cp_async_wait<0>();
  finish_group<NR, SW, NB>(p, acc, grp, n0, col);
}

// ---------------------------------------------------------------------------
// [M,K] MX weights: mxfp4 (A16), mxfp4/a4, mxfp4/a8, mxfp4/f8
// ---------------------------------------------------------------------------
template <int DT, int NR>
struct KmT {
  static constexpr int SW = 16;                        // weight rows per warp
  static constexpr int XBITS = x_is_half(DT) ? 16 : (x_is_e4m3(DT) ? 8 : 4);
  static constexpr int RSTRIDE = 80;                   // 64 bytes of a row + 16: conflict-free lane reads
  static constexpr int SC_OFF = SW * RSTRIDE;          // 16 rows x 4 block scales
  static constexpr int X_OFF = SC_OFF + SW * 4;        // [NR rows][4 t][4 blocks][16 B]
  static constexpr int XS_OFF = X_OFF + NR * 256;      // [NR][4 block scales] (a4/a8)
  static constexpr int STAGE = (XS_OFF + NR * 4 + 15) / 16 * 16;
};

template <int DT, int NR>
__global__ void __launch_bounds__(kMThreads, kMCtasPerSm) gemv_mma_km_kernel(MmaParams p) {
  using T = KmT<DT, NR>;
  constexpr int SW = T::SW, STAGE = T::STAGE, XBITS = T::XBITS;
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.z * NR;
  int u0, u1;
  run_of(blockIdx.x, gridDim.x, p.units, u0, u1);
  if (u0 >= u1) return;   // CTA-uniform

  const uint32_t ring = (uint32_t)__cvta_generic_to_shared(smem) + (uint32_t)(warp * kStages * STAGE);
  const int kb = p.K / 32;                 // blocks (and scales) per weight row
  const size_t rowb = (size_t)p.K / 2;     // bytes per weight row
  const uint8_t* W = static_cast<const uint8_t*>(p.W);
  const uint8_t* X = static_cast<const uint8_t*>(p.X);

  // unit u: group u / ks (128 weight rows, 16 per warp), blocks 4 (u % ks) .. +3
  auto issue = [&](int grp, int j, int stage) {
    const int blk0 = 4 * j;
    const uint32_t st = ring + (uint32_t)(stage * STAGE);
    const int mrow0 = (grp * kMWarps + warp) * SW;
    // weights: 16 rows x 64 bytes = 64 chunks of 16 bytes, two per lane
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int q = 2 * lane + h, row = q >> 2, cch = q & 3;
      const int m = mrow0 + row;
      const bool ok = m < p.M;
      cp_async16(st + (uint32_t)(row * T::RSTRIDE + cch * 16),
                 ok ? W + (size_t)m * rowb + (size_t)blk0 * 16 + cch * 16 : W, ok ? 16u : 0u);
    }
    if (lane < SW) {   // the 4 block scales of row `lane`
      const int m = mrow0 + lane;
      const bool ok = m < p.M;
      cp_async4(st + T::SC_OFF + lane * 4, ok ? p.wscale + (size_t)m * kb + blk0 : p.wscale, ok ? 4u : 0u);
    }
    if (g < NR) {      // X row n0 + g: the lane's 8 K elements of each block
      const bool ok = n0 + g < p.N;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const size_t e = (size_t)(ok ? n0 + g : 0) * p.K + (size_t)(blk0 + b) * 32 + 8 * t;
        const uint32_t dst = st + T::X_OFF + (uint32_t)(((g * 4 + t) * 4 + b) * 16);
        if constexpr (XBITS == 16) cp_async16(dst, X + e * 2, ok ? 16u : 0u);
        else if constexpr (XBITS == 8) cp_async8(dst, X + e, ok ? 8u : 0u);
        else cp_async4(dst, X + e / 2, ok ? 4u : 0u);
      }
    }
    if constexpr (x_scaled(DT)) {
      if (g == 0) {    // the X block scales of C columns 2t, 2t+1
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int n = 2 * t + h;
          if (n < NR) {
            const bool ok = n0 + n < p.N;
            cp_async4(st + T::XS_OFF + n * 4, ok ? p.xscale + (size_t)(n0 + n) * kb + blk0 : p.xscale,
                      ok ? 4u : 0u);
          }
        }
      }
    }
  };

  float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
  auto compute = [&](int stage) {
    const uint32_t st = ring + (uint32_t)(stage * STAGE);
    const uint32_t scg = lds32(st + T::SC_OFF + g * 4), scg8 = lds32(st + T::SC_OFF + (g + 8) * 4);
    uint32_t xs0w = 0x7F7F7F7Fu, xs1w = 0x7F7F7F7Fu;   // 2^0 per block where X has no scales
    if constexpr (x_scaled(DT)) {
      if (2 * t < NR) xs0w = lds32(st + T::XS_OFF + (2 * t) * 4);
      if (2 * t + 1 < NR) xs1w = lds32(st + T::XS_OFF + (2 * t + 1) * 4);
    }
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      // xf[i] = x[8t + 2i], x[8t + 2i + 1] of block b as f16 (exact); zero past NR rows
      uint32_t xf[4] = {0u, 0u, 0u, 0u};
      if (g < NR) {
        const uint32_t xa = st + T::X_OFF + (uint32_t)(((g * 4 + t) * 4 + b) * 16);
        if constexpr (XBITS == 16) {
          const uint4 v = lds128(xa);
          xf[0] = v.x;
          xf[1] = v.y;
          xf[2] = v.z;
          xf[3] = v.w;
        } else if constexpr (XBITS == 8) {
          const uint2 v = lds64(xa);
          xf[0] = cvt_e4m3x2(v.x);
          xf[1] = cvt_e4m3x2(v.x >> 16);
          xf[2] = cvt_e4m3x2(v.y);
          xf[3] = cvt_e4m3x2(v.y >> 16);
        } else {
          e2m1x8_to_f16x2(lds32(xa), xf);
        }
      }
      uint32_t hg[4], hg8[4];   // rows g and g+8: k pairs (8t, 8t+1) .. (8t+6, 8t+7) of block b
      e2m1x8_to_f16x2(lds32(st + (uint32_t)(g * T::RSTRIDE + b * 16 + 4 * t)), hg);
      e2m1x8_to_f16x2(lds32(st + (uint32_t)((g + 8) * T::RSTRIDE + b * 16 + 4 * t)), hg8);
      float tb[4] = {0.f, 0.f, 0.f, 0.f};
      mma_f16(tb, hg[0], hg8[0], hg[1], hg8[1], xf[0], xf[1]);
      mma_f16(tb, hg[2], hg8[2], hg[3], hg8[3], xf[2], xf[3]);
      const float sg = dec_ue8m0((scg >> (8 * b)) & 0xFFu), sg8 = dec_ue8m0((scg8 >> (8 * b)) & 0xFFu);
      float xs0 = 1.f, xs1 = 1.f;
      if constexpr (x_scaled(DT)) {
        xs0 = dec_ue8m0((xs0w >> (8 * b)) & 0xFFu);
        xs1 = dec_ue8m0((xs1w >> (8 * b)) & 0xFFu);
      }
      acc[0][0] = fmaf(tb[0], sg * xs0, acc[0][0]);
      acc[0][1] = fmaf(tb[1], sg * xs1, acc[0][1]);
      acc[0][2] = fmaf(tb[2], sg8 * xs0, acc[0][2]);
      acc[0][3] = fmaf(tb[3], sg8 * xs1, acc[0][3]);
    }
  };
  // C row g is weight row g of the warp's 16, row g+8 is g + 8
  auto col = [&](int, int h) { return g + 8 * h; };

  int igrp = u0 / p.ks, ij = u0 - igrp * p.ks;   // next unit to copy
  int grp = igrp, cgrp = igrp, cj = ij;            // group in acc; unit to multiply
#pragma unroll
  for (int q = 0; q < kStages - 1; ++q) {
    if (u0 + q < u1) {
      issue(igrp, ij, q);
      next_unit(igrp, ij, p.ks);
    }
    cp_async_commit();
  }
  int stage = 0;
  for (int u = u0; u < u1; ++u) {
    cp_async_wait<kStages - 2>();
    // every lane's copies of unit u have landed (lanes read each other's rows),
    // and every lane is done with the stage read in the previous step
    __syncwarp();
    if (u + kStages - 1 < u1) {
      issue(igrp, ij, stage == 0 ? kStages - 1 : stage - 1);
      next_unit(igrp, ij, p.ks);
    }
    cp_async_commit();
    if (cgrp != grp) {
      finish_group<NR, SW, 1>(p, acc, grp, n0, col);
      grp = cgrp;
    }
    compute(stage);
    next_unit(cgrp, cj, p.ks);
    stage = stage == kStages - 1 ? 0 : stage + 1;
  }
  cp_async_wait<0>();
  finish_group<NR, SW, 1>(p, acc, grp, n0, col);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
bool mn_kind(int dt) { return dt == kFP16 || dt == kINT8 || dt == kFP8 || dt == kF8F8; }

int mma_nr(int N) { return N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : 8; }

struct MmaGeom {
  int sw, ngroups, ks, units, nr, nrowblk;
  size_t stage;
};

MmaGeom mma_geom(int dt, int N, int K, int M) {
  MmaGeom g;
  g.nr = mma_nr(N);
  g.nrowblk = (N + g.nr - 1) / g.nr;
  if (w_is_mx(dt)) {
    g.sw = 16;
    g.ks = K / 128;
    const size_t s = 16 * 80 + 16 * 4 + (size_t)g.nr * 256 + (size_t)g.nr * 4;
    g.stage = (s + 15) / 16 * 16;
  } else {
    g.sw = dt == kFP16 ? 64 : 128;
    g.ks = (K + 15) / 16;
    g.stage = 4 * 32 * 16 + 32 * 8;
  }
  const int cols = kMWarps * g.sw;   // output columns of a group
  g.ngroups = (M + cols - 1) / cols;
  g.units = g.ngroups * g.ks;
  return g;
}

int mma_grid(const MmaGeom& g, int num_sms) {
  long G = (long)kMCtasPerSm * (num_sms > 0 ? num_sms : 148);
  if (G > kMaxMCtas) G = kMaxMCtas;
  if (G > g.units) G = g.units;
  return G < 1 ? 1 : (int)G;
}

size_t mma_smem(const MmaGeom& g) { return (size_t)kMWarps * kStages * g.stage; }

template <int DT, int NR>
cudaError_t launch_mma_nr(const MmaParams& p, int G, int nrowblk, size_t smem, cudaStream_t st) {
  auto launch = [&](auto k) -> cudaError_t {
    // opt in above 47 KiB: the 48 KiB default also holds the kernel's static flag
    if (smem > 47 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    k<<<dim3(G, 1, nrowblk), kMThreads, smem, st>>>(p);
    return cudaGetLastError();
  };
  if constexpr (w_is_mx(DT)) return launch(gemv_mma_km_kernel<DT, NR>);
  else return launch(gemv_mma_mn_kernel<DT, NR>);
}

template <int DT>
cudaError_t launch_mma_dt(const MmaParams& p, int nr, int G, int nrowblk, size_t smem, cudaStream_t st) {
  switch (nr) {
    case 1: return launch_mma_nr<DT, 1>(p, G, nrowblk, smem, st);
    case 2: return launch_mma_nr<DT, 2>(p, G, nrowblk, smem, st);
    case 4: return launch_mma_nr<DT, 4>(p, G, nrowblk, smem, st);
    default: return launch_mma_nr<DT, 8>(p, G, nrowblk, smem, st);
  }
}

bool aligned_to(const void* ptr, unsigned a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

}  // namespace

bool mma_supported(int dt, int N, int K, int M) {
  if (N < 1 || N > 16 || K < 1 || M < 1) return false;
  if (w_is_mx(dt)) {
    // steps of 4 blocks: whole 64-byte row pieces and 4-byte groups of scales
    if (K % 128 != 0) return false;
  } else if (mn_kind(dt)) {
    // every lane's 16-byte chunk of a row is whole, and X's 4-element groups too
    if (K % 4 != 0 || ((long)M * (dt == kFP16 ? 2 : 1)) % 16 != 0) return false;
  } else {
    return false;   // i8i8 (exact int32) and f4f4 stay on the CUDA-core kernels
  }
  const MmaGeom g = mma_geom(dt, N, K, M);
  if ((size_t)g.nrowblk * g.ngroups * sizeof(unsigned) > kMCounterBytes) return false;
  // the device partition arithmetic is 32-bit: (units + 1) * grid < 2^32
  if (((uint64_t)g.units + 1) * kMaxMCtas >= (1ull << 32)) return false;
  return mma_smem(g) <= kMaxMSmem;
}

size_t mma_workspace(int dt, int N, int K, int M) {
  const MmaGeom g = mma_geom(dt, N, K, M);
  const size_t tile = (size_t)kMWarps * g.nr * g.sw;
  return kMCounterBytes + (size_t)g.nrowblk * (g.ngroups + kMaxMCtas) * tile * sizeof(float);
}

cudaError_t launch_mma(const RunArgs& a) {
  if (!mma_supported(a.dt, a.N, a.K, a.M)) return cudaErrorInvalidValue;
  if (!a.ws || a.ws_bytes < mma_workspace(a.dt, a.N, a.K, a.M)) return cudaErrorInvalidValue;
  // cp.async sources: whole 16-byte row chunks of the weights; X in the width of
  // one copy (8 or 4 bytes for [K,M] kinds, 16 / 8 / 4 for the MX kinds)
  if (!aligned_to(a.W, 16)) return cudaErrorInvalidValue;
  const unsigned xal = w_is_mx(a.dt) ? (x_is_half(a.dt) ? 16 : x_is_e4m3(a.dt) ? 8 : 4) : (x_is_half(a.dt) ? 8 : 4);
  if (!aligned_to(a.X, xal)) return cudaErrorInvalidValue;
  if (w_is_mx(a.dt) && (!aligned_to(a.wscale, 4) || (x_scaled(a.dt) && !aligned_to(a.xscale, 4))))
    return cudaErrorInvalidValue;
  const MmaGeom g = mma_geom(a.dt, a.N, a.K, a.M);
  const int G = mma_grid(g, a.num_sms);
  MmaParams p;
  p.X = a.X;
  p.W = a.W;
  p.Y = a.Y;
  p.xscale = a.xscale;
  p.wscale = a.wscale;
  p.N = a.N;
  p.K = a.K;
  p.M = a.M;
  p.ngroups = g.ngroups;
  p.ks = g.ks;
  p.units = g.units;
  p.counters = reinterpret_cast<unsigned*>(a.ws);
  p.part = reinterpret_cast<float*>(static_cast<char*>(a.ws) + kMCounterBytes);
  const size_t smem = mma_smem(g);
  switch (a.dt) {
    case kFP16: return launch_mma_dt<kFP16>(p, g.nr, G, g.nrowblk, smem, a.stream);
    case kINT8: return launch_mma_dt<kINT8>(p, g.nr, G, g.nrowblk, smem, a.stream);
    case kFP8: return launch_mma_dt<kFP8>(p, g.nr, G, g.nrowblk, smem, a.stream);
    case kF8F8: return launch_mma_dt<kF8F8>(p, g.nr, G, g.nrowblk, smem, a.stream);
    case kMXFP4: return launch_mma_dt<kMXFP4>(p, g.nr, G, g.nrowblk, smem, a.stream);
    case kMX4X4: return launch_mma_dt<kMX4X4>(p, g.nr, G, g.nrowblk, smem, a.stream);
    case kMX8X4: return launch_mma_dt<kMX8X4>(p, g.nr, G, g.nrowblk, smem, a.stream);
    case kF8X4: return launch_mma_dt<kF8X4>(p, g.nr, G, g.nrowblk, smem, a.stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mlpg
