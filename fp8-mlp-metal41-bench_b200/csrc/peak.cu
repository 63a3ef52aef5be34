// peak.cu -- pure-compute tcgen05 peak probe (the B200 counterpart of the
// reference's tune/peak.metal + tune/peak.swift).
//
// tune/peak.metal:29-87 runs matmul2d R times on operands resident in
// threadgroup memory, so the loop has no DRAM traffic.  Here every CTA (one
// per SM, or one CTA pair per two SMs for cta_group::2) fills a 128-row A
// tile and an N-row B tile in shared memory once, then one thread issues
// `reps` x 4 tcgen05.mma (one 128-byte K stage each time) into a TMEM
// accumulator and waits for them with tcgen05.commit.  The host times the
// launch with CUDA events; dense FLOP/s (OP/s for kind::i8) =
// 2 * M * N * K_mma * 4 * reps * (CTAs or pairs) / time.
//
// Probe kinds (gemm_peak_probe): 0 f16, 1 i8, 2 f8f6f4 (E4M3), 3 mxf8f6f4
// (E4M3 x E2M1, UE8M0 block 32), 4 mxf4 (E2M1 x E2M1, block 32), and
// 5 f16 / 6 i8 / 7 f8f6f4 on CTA pairs (cta_group::2, M = 256).  Kinds
// 8 f16 / 9 i8 / 10 f8f6f4 are the pairs again with B read MN-major (the
// instruction descriptor's transpose-B bit, 128-byte swizzle atoms along N),
// the operand layout of the [K,M] weights in the GEMM's pair kernel.  Kinds
// 11 mxf8f6f4 / 12 mxf4 are the block-scaled kinds on CTA pairs (K-major B,
// unit scale cells copied to TMEM once), and 13 / 14 the same with the GEMM's
// per-stage scale-cell copies issued before each stage's MMAs (3 for
// mxf8f6f4, 6 for mxf4: one 32x128b.warpx4 copy per 128 rows x 4 scales of X
// and of the pair's 256 W columns), into a ring of 4 TMEM slots.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"

namespace mlpg {

namespace {

constexpr int kPeakN = 256;
constexpr int kPeakThreads = 128;
constexpr int kA = 128 * 128;             // A tile bytes (128 rows x 128 B)
constexpr int kB = kPeakN * 128;          // B tile bytes (256 rows x 128 B)
constexpr int kSfOff = kA + kB;           // 512 B of unit scale factors
constexpr int kBarOff = kSfOff + 512;
constexpr int kPeakSmem = kBarOff + 64 + 1024;

template <int KIND, bool PAIR, bool BMN = false>
constexpr uint32_t peak_idesc() {
  constexpr uint32_t m = PAIR ? 256u : 128u;   // a pair computes 256 rows; each CTA holds N/2 of B
  constexpr uint32_t n = (uint32_t)kPeakN;
  constexpr uint32_t tb = BMN ? (1u << 16) : 0u;   // B MN-major
  if constexpr (KIND == kKindF16) return (1u << 4) | tb | ((n >> 3) << 17) | ((m >> 4) << 24);
  if constexpr (KIND == kKindI8)
    return (2u << 4) | (1u << 7) | (1u << 10) | tb | ((n >> 3) << 17) | ((m >> 4) << 24);
  if constexpr (KIND == kKindF8F6F4) return (1u << 4) | tb | ((n >> 3) << 17) | ((m >> 4) << 24);
  if constexpr (KIND == kKindMxF8F6F4)
    return (0u << 7) | (5u << 10) | ((n >> 3) << 17) | (1u << 23) | ((m >> 4) << 24);
  return (1u << 7) | (1u << 10) | ((n >> 3) << 17) | (1u << 23) | ((m >> 4) << 24);   // mxf4
}

template <int KIND, bool PAIR, bool BMN = false, bool SFCP = false>
__global__ void __launch_bounds__(kPeakThreads, 1) peak_kernel(int reps, float* sink, int* dev_err) {
  static_assert(!BMN || PAIR, "MN-major B: pair probes");
  static_assert(!SFCP || (PAIR && KIND >= kKindMxF8F6F4), "per-stage scale copies: block-scaled pairs");
  // MN-major B as the pair kernel lays it out: boxes of (128 bytes of N) x
  // (one 128-byte K stage), the boxes kBox bytes apart (the descriptor's
  // leading-dimension offset); one MMA's K slice starts kAdv bytes further on
  constexpr int kEs = KIND == kKindF16 ? 2 : 1;
  constexpr uint32_t kBoxMn = 128 / kEs;                     // N elements per box
  constexpr uint32_t kBoxK = 128 / kEs;                      // K elements per stage
  constexpr uint32_t kBox = kBoxK * 128;                     // bytes per box
  constexpr uint32_t kAdv = (32 / kEs) * 128;                // K rows of one MMA x 128 B
  static_assert(!BMN || (kPeakN / 2 / kBoxMn) * kBox <= (uint32_t)kB, "B boxes fit the B tile");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* done = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint32_t* tbase = reinterpret_cast<uint32_t*>(smem + kBarOff + 8);
  int* abort_flag = reinterpret_cast<int*>(smem + kBarOff + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  AbortCtl ctl{dev_err, abort_flag};

  // small finite values in every format: bytes 0x00..0x33 (cf. tune/peak.metal:45-47)
  for (int i = threadIdx.x; i < (kA + kB) / 4; i += kPeakThreads) {
    const uint32_t b = ((uint32_t)i * 37u + 11u) & 0x33u;
    reinterpret_cast<uint32_t*>(smem)[i] = b | (b << 8) | (b << 16) | (b << 24);
  }
  if (threadIdx.x < 32) reinterpret_cast<uint4*>(smem + kSfOff)[threadIdx.x] =
      make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  fence_proxy_async_smem();
  constexpr uint32_t cols = PAIR ? 2 * kPeakN : 512;   // accumulator (+ scale factors)
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tbase, cols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tbase, cols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tbase;
  const bool leader = !PAIR || cluster_ctarank() == 0;

  if (warp == 0 && lane == 0 && leader) {
    constexpr uint32_t idesc = peak_idesc<KIND, PAIR, BMN>();
    const uint32_t a = smem_u32(smem), b = a + kA, sf = a + kSfOff;
    // scale cells: slot q of 4 holds 2 cells x (4 A + 8 B columns) after the accumulator
    constexpr int kCells = KIND == kKindMxF4 ? 2 : 1;
    auto slot = [&](int q) { return tmem + kPeakN + (uint32_t)(q * 24); };
    auto copy_cells = [&](uint32_t base) {
#pragma unroll
      for (int g = 0; g < kCells; ++g) {
        const uint32_t t = base + g * 12;
        if constexpr (PAIR) {
          tc_cp_pair_32x128b_warpx4(t, sdesc_plain(sf, 0, 128));
          for (int c = 0; c < kPeakN / 128; ++c) tc_cp_pair_32x128b_warpx4(t + 4 + 4 * c, sdesc_plain(sf, 0, 128));
        } else {
          tc_cp_32x128b_warpx4(t, sdesc_plain(sf, 0, 128));
          for (int c = 0; c < kPeakN / 128; ++c) tc_cp_32x128b_warpx4(t + 4 + 4 * c, sdesc_plain(sf, 0, 128));
        }
      }
    };
    if constexpr (KIND >= kKindMxF8F6F4) copy_cells(slot(0));
    for (int r = 0; r < reps; ++r) {
      const uint32_t sfa_t = slot(SFCP ? (r & 3) : 0), sfb_t = sfa_t + 4;
      if constexpr (SFCP) copy_cells(sfa_t);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = sdesc_sw128(a + kk * 32, 16, 1024);
        const uint64_t bd = BMN ? sdesc_sw128(b + kk * kAdv, kBox, 1024) : sdesc_sw128(b + kk * 32, 16, 1024);
        const uint32_t acc = (r | kk) != 0 ? 1u : 0u;
        // the cell of this MMA's K slice (mxf4: two MMAs per cell, as in the GEMM)
        const uint32_t cell = KIND == kKindMxF4 ? (uint32_t)(kk / 2) * 12u : 0u;
        if constexpr (PAIR && KIND >= kKindMxF8F6F4)
          tc_mma_pair_bs<KIND>(tmem, ad, bd, idesc, acc, sfa_t + cell, sfb_t + cell);
        else if constexpr (PAIR) tc_mma_pair<KIND>(tmem, ad, bd, idesc, acc);
        else if constexpr (KIND >= kKindMxF8F6F4) tc_mma_bs<KIND>(tmem, ad, bd, idesc, acc, sfa_t + cell, sfb_t + cell);
        else tc_mma<KIND>(tmem, ad, bd, idesc, acc);
      }
    }
    if constexpr (PAIR) tc_commit_pair(done, 0x3); else tc_commit(done);
  }
  __syncwarp();
  // every thread waits for the MMAs (bounded), then one value is kept alive
  const bool ok = mbar_wait(done, 0, ctl, 0x800);
  tc_fence_after();
  if (warp == 0) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tmem, r);
    tmem_ld_wait();
    if (lane == 0 && ok) sink[blockIdx.x] = __uint_as_float(r[0]);
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync(); else __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, cols); else tmem_dealloc(tmem, cols);
  }
}

template <int KIND, bool PAIR, bool BMN = false, bool SFCP = false>
cudaError_t launch_one(int reps, int ctas, float* sink, int* dev_err, cudaStream_t st) {
  auto k = peak_kernel<KIND, PAIR, BMN, SFCP>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeakSmem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kPeakThreads);
  cfg.dynamicSmemBytes = kPeakSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, reps, sink, dev_err);
}

}  // namespace

// K elements per tcgen05.mma by probe kind
static int peak_kmma(int kind) {
  switch (kind) {
    case 0: case 5: case 8: return 16;
    case 4: case 12: case 14: return 64;
    default: return 32;
  }
}

double peak_flops_per_launch(int kind, int reps, int ctas) {
  const bool pair = kind >= 5;
  const double m = pair ? 256.0 : 128.0, n = kPeakN;
  const double units = pair ? ctas / 2 : ctas;
  return 2.0 * m * n * peak_kmma(kind) * 4.0 * reps * units;
}

cudaError_t launch_peak(int kind, int reps, int ctas, float* sink, int* dev_err, cudaStream_t st) {
  switch (kind) {
    case 0: return launch_one<kKindF16, false>(reps, ctas, sink, dev_err, st);
    case 1: return launch_one<kKindI8, false>(reps, ctas, sink, dev_err, st);
    case 2: return launch_one<kKindF8F6F4, false>(reps, ctas, sink, dev_err, st);
    case 3: return launch_one<kKindMxF8F6F4, false>(reps, ctas, sink, dev_err, st);
    case 4: return launch_one<kKindMxF4, false>(reps, ctas, sink, dev_err, st);
    case 5: return launch_one<kKindF16, true>(reps, ctas, sink, dev_err, st);
    case 6: return launch_one<kKindI8, true>(reps, ctas, sink, dev_err, st);
    case 7: return launch_one<kKindF8F6F4, true>(reps, ctas, sink, dev_err, st);
    case 8: return launch_one<kKindF16, true, true>(reps, ctas, sink, dev_err, st);
    case 9: return launch_one<kKindI8, true, true>(reps, ctas, sink, dev_err, st);
    case 10: return launch_one<kKindF8F6F4, true, true>(reps, ctas, sink, dev_err, st);
    case 11: return launch_one<kKindMxF8F6F4, true>(reps, ctas, sink, dev_err, st);
    case 12: return launch_one<kKindMxF4, true>(reps, ctas, sink, dev_err, st);
    case 13: return launch_one<kKindMxF8F6F4, true, false, true>(reps, ctas, sink, dev_err, st);
    case 14: return launch_one<kKindMxF4, true, false, true>(reps, ctas, sink, dev_err, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mlpg
