// gemm_tc.cu -- tcgen05 tensor-core GEMM for sm_100a.
//
// Replaces the reference's matmul2d kernels (fp8_mlp.metal:58-444), which
// hand the whole K loop to Apple's closed MetalPerformancePrimitives.  Here
// the loop is explicit and Blackwell-native:
//
//   warp 0      TMA producer: X and W tiles -> a STAGES-deep shared-memory
//               ring (128-byte swizzle), completion on "full" mbarriers
//   warp 1      TMEM allocator + single-thread MMA issuer: tcgen05.mma into a
//               double-buffered TMEM accumulator, tcgen05.commit frees ring
//               slots ("empty") and hands finished tiles to the epilogue
//   warp 2      (block-scaled kinds) UE8M0 scale-factor stager
//   warps 4-7   epilogue: tcgen05.ld TMEM -> registers -> Y, one TMEM lane
//               quadrant (32 output rows) per warp
//
// The grid is persistent (one CTA per SM); output tiles are BM=128 rows of
// Y by BN (128 or 256) columns.  X is always K-major.  W is MN-major for
// the [K,M] dtypes (fp16, i8i8, f8f8: the instruction descriptor's
// "transpose B" bit) and K-major for the [M,K] mxfp4 family.
//
// Every mbarrier wait is bounded (ptx.cuh); on expiry the kernel records
// an error word, lets in-flight TMA copies land, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "formats.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace mlpg {

namespace {

constexpr int kBM = 128;
constexpr int kThreads = 256;
constexpr int kRowBytes = 128;   // bytes of K per operand row per stage (one swizzle row)

// Per-dtype kernel traits.
template <int DT>
struct Traits;

template <>
struct Traits<kFP16> {
  static constexpr int kind = kKindF16;
  static constexpr int a_bits = 16, b_bits = 16;
  static constexpr bool b_mn = true, out_int = false, scaled = false;
  static constexpr uint32_t a_fmt = 0, b_fmt = 0, c_fmt = 1;  // F16, F16 -> F32
};
template <>
struct Traits<kI8I8> {
  static constexpr int kind = kKindI8;
  static constexpr int a_bits = 8, b_bits = 8;
  static constexpr bool b_mn = true, out_int = true, scaled = false;
  static constexpr uint32_t a_fmt = 1, b_fmt = 1, c_fmt = 2;  // S8, S8 -> S32
};
template <>
struct Traits<kF8F8> {
  static constexpr int kind = kKindF8F6F4;
  static constexpr int a_bits = 8, b_bits = 8;
  static constexpr bool b_mn = true, out_int = false, scaled = false;
  static constexpr uint32_t a_fmt = 0, b_fmt = 0, c_fmt = 1;  // E4M3, E4M3 -> F32
};

struct TcParams {
  void* Y;
  int N, K, M;
  int tiles_m, tiles_n, num_kb;
  int* dev_err;
};

template <int DT, int BN, int STAGES>
struct Cfg {
  using T = Traits<DT>;
  static constexpr int A_BYTES = kBM * kRowBytes;            // 16 KB
  static constexpr int B_BYTES = BN * kRowBytes;             // 16 / 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int K_PER_STAGE = kRowBytes * 8 / T::a_bits;  // elements
  static constexpr int MMA_K_BYTES = 32;                     // K bytes per tcgen05.mma
  static constexpr int MMAS_PER_STAGE = kRowBytes / MMA_K_BYTES;  // 4
  // MN-major B: one TMA box is K_PER_STAGE rows x 128 bytes of MN
  static constexpr int B_BOX_MN = kRowBytes * 8 / T::b_bits; // MN elements per box
  static constexpr int B_BOXES = T::b_mn ? BN / B_BOX_MN : 1;
  static constexpr int B_BOX_BYTES = T::b_mn ? K_PER_STAGE * kRowBytes : B_BYTES;
  // descriptor strides
  static constexpr uint32_t B_LBO = T::b_mn ? (uint32_t)B_BOX_BYTES : 16u;
  static constexpr uint32_t B_ADV = T::b_mn ? (uint32_t)(MMA_K_BYTES * 8 / T::b_bits) * kRowBytes
                                            : (uint32_t)MMA_K_BYTES;
  static constexpr int ACC_COLS = BN;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;    // + barriers + alignment slack
  static constexpr uint32_t IDESC =
      (T::c_fmt << 4) | (T::a_fmt << 7) | (T::b_fmt << 10) | (0u << 15) |
      ((T::b_mn ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
  static_assert(BN % 16 == 0 && BN <= 256, "UMMA N");
  static_assert(!T::b_mn || BN % B_BOX_MN == 0, "MN-major B tile must be whole swizzle atoms");
};

struct Bars {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int& tm, int& tn) {
  tm = tile % tiles_m;
  tn = tile / tiles_m;
}

template <int DT, int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   TcParams p) {
  using C = Cfg<DT, BN, STAGES>;
  using T = typename C::T;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + C::BAR_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;
  AbortCtl ctl{p.dev_err, &bars->abort_flag};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 4 * 32);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
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
    uint32_t filled_parity[8];
    bool filled[8];
    for (int s = 0; s < STAGES; ++s) filled[s] = false, filled_parity[s] = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, tm, tn);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&bars->empty[stage], phase ^ 1u, ctl, 0x100 + stage)) { ok = false; break; }
        unsigned char* a_dst = smem + stage * C::STAGE_BYTES;
        unsigned char* b_dst = a_dst + C::A_BYTES;
        mbar_arrive_expect_tx(&bars->full[stage], C::STAGE_BYTES);
        // A tile: x in elements of the map (bytes for 8/4-bit maps)
        tma_load_2d(a_dst, &tmA, &bars->full[stage], kb * (T::a_bits == 16 ? C::K_PER_STAGE : kRowBytes),
                    tm * kBM);
        if constexpr (T::b_mn) {
#pragma unroll
          for (int j = 0; j < C::B_BOXES; ++j)
            tma_load_2d(b_dst + j * C::B_BOX_BYTES, &tmB, &bars->full[stage],
                        tn * BN + j * C::B_BOX_MN, kb * C::K_PER_STAGE);
        } else {
          tma_load_2d(b_dst, &tmB, &bars->full[stage], kb * kRowBytes, tn * BN);
        }
        filled[stage] = true;
        filled_parity[stage] = phase;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
    if (!ok) {
      // let copies already in flight land before the CTA exits
      for (int s = 0; s < STAGES; ++s) {
        if (!filled[s]) continue;
        const uint32_t a = smem_u32(&bars->full[s]);
        const unsigned long long t0 = global_ns();
        while (!mbar_try_wait(a, filled_parity[s]) && global_ns() - t0 < kWaitTimeoutNs) {}
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------ MMA issuer --------------------------------
    uint32_t stage = 0, phase = 0;
    int local = 0;
    bool ok = true;
    const uint32_t smem_base = smem_u32(smem);
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t acc_par = (uint32_t)(local >> 1) & 1u;
      if (!mbar_wait(&bars->acc_empty[buf], acc_par ^ 1u, ctl, 0x200 + buf)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(buf * C::ACC_COLS);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&bars->full[stage], phase, ctl, 0x300 + stage)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_base + stage * C::STAGE_BYTES;
        const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < C::MMAS_PER_STAGE; ++kk) {
          const uint64_t adesc = sdesc_sw128(a_addr + kk * C::MMA_K_BYTES, 16, 1024);
          const uint64_t bdesc = sdesc_sw128(b_addr + kk * C::B_ADV, C::B_LBO, 1024);
          tc_mma<T::kind>(d_tmem, adesc, bdesc, C::IDESC, (kb | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&bars->empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      tc_commit(&bars->acc_full[buf]);
    }
  } else if (warp >= 4) {
    // ------------------------------ epilogue ----------------------------------
    const int q = warp - 4;  // TMEM lane quadrant == warp % 4
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, tm, tn);
      const int buf = local & 1;
      const uint32_t acc_par = (uint32_t)(local >> 1) & 1u;
      const bool got = mbar_wait(&bars->acc_full[buf], acc_par, ctl, 0x400 + buf);
      if (!__all_sync(0xffffffffu, got)) break;   // the warp leaves together
      __syncwarp();                               // tcgen05.ld is .sync.aligned
      tc_fence_after();
      const int row = tm * kBM + q * 32 + lane;
      const int col0 = tn * BN;
      const bool row_ok = row < p.N;
      uint32_t* yrow = reinterpret_cast<uint32_t*>(p.Y) + (size_t)row * p.M;
      const bool vec_ok = (p.M % 4) == 0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * C::ACC_COLS + c * 32), r);
        tmem_ld_wait();
        const int cb = col0 + c * 32;
        if (row_ok) {
          if (vec_ok && cb + 32 <= p.M) {
            uint4* dst = reinterpret_cast<uint4*>(yrow + cb);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_uint4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
          } else {
#pragma unroll
            for (int v = 0; v < 32; ++v)
              if (cb + v < p.M) yrow[cb + v] = r[v];
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->acc_empty[buf]);
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

// ----------------------------------------------------------------------------
// host side: tensor maps through the driver entry point (no libcuda link)
// ----------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D row-major map: `inner` elements per row (contiguous), `outer` rows.
bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType ty, int elem_bytes,
              uint64_t inner, uint64_t outer, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, ty, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int DT, int BN, int STAGES>
cudaError_t launch_cfg(const RunArgs& a) {
  using C = Cfg<DT, BN, STAGES>;
  using T = typename C::T;
  CUtensorMap tmA, tmB;
  const CUtensorMapDataType ty8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  bool ok;
  if constexpr (T::a_bits == 16) {
    ok = make_map(&tmA, a.X, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)a.K, (uint64_t)a.N,
                  C::K_PER_STAGE, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    const uint64_t row_bytes = (uint64_t)a.K * T::a_bits / 8;
    ok = make_map(&tmA, a.X, ty8, 1, row_bytes, (uint64_t)a.N, kRowBytes, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (!ok) return cudaErrorInvalidValue;
  if constexpr (T::b_mn) {
    const int es = T::b_bits / 8;
    ok = make_map(&tmB, a.W, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : ty8, es, (uint64_t)a.M,
                  (uint64_t)a.K, C::B_BOX_MN, C::K_PER_STAGE, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    const uint64_t row_bytes = (uint64_t)a.K * T::b_bits / 8;
    ok = make_map(&tmB, a.W, ty8, 1, row_bytes, (uint64_t)a.M, kRowBytes, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (!ok) return cudaErrorInvalidValue;

  TcParams p;
  p.Y = a.Y;
  p.N = a.N;
  p.K = a.K;
  p.M = a.M;
  p.tiles_m = (a.N + kBM - 1) / kBM;
  p.tiles_n = (a.M + BN - 1) / BN;
  p.num_kb = (a.K + C::K_PER_STAGE - 1) / C::K_PER_STAGE;
  p.dev_err = a.dev_err;
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < a.num_sms ? tiles : a.num_sms;
  auto k = tc_gemm_kernel<DT, BN, STAGES>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  k<<<grid, kThreads, C::SMEM_BYTES, a.stream>>>(tmA, tmB, p);
  return cudaGetLastError();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool tc_supported(int dt, int bn, int N, int K, int M) {
  if (bn != 128 && bn != 256) return false;
  if (N <= 0 || K <= 0 || M <= 0) return false;
  switch (dt) {
    case kFP16: return K % 8 == 0 && M % 8 == 0;
    case kI8I8:
    case kF8F8: return K % 16 == 0 && M % 16 == 0;
    default: return false;
  }
}

size_t tc_workspace(int dt, int bn, int N, int K, int M) {
  (void)dt; (void)bn; (void)N; (void)K; (void)M;
  return 0;
}

int tc_launches(int dt) {
  (void)dt;
  return 1;
}

cudaError_t launch_tc(const RunArgs& a, int bn) {
  if (!tc_supported(a.dt, bn, a.N, a.K, a.M)) return cudaErrorInvalidValue;
  if (!aligned16(a.X) || !aligned16(a.W) || !aligned16(a.Y)) return cudaErrorInvalidValue;
  switch (a.dt) {
    case kFP16: return bn == 256 ? launch_cfg<kFP16, 256, 4>(a) : launch_cfg<kFP16, 128, 6>(a);
    case kI8I8: return bn == 256 ? launch_cfg<kI8I8, 256, 4>(a) : launch_cfg<kI8I8, 128, 6>(a);
    case kF8F8: return bn == 256 ? launch_cfg<kF8F8, 256, 4>(a) : launch_cfg<kF8F8, 128, 6>(a);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mlpg
