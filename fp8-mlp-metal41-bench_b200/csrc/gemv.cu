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

// Decode `E` weights from an aligned register chunk (raw bytes of one row).
template <int DT, int E, int LW>
__device__ __forceinline__ void decode_w_chunk(const uint32_t (&raw)[LW / 4], float (&w)[E]) {
  const uint8_t* b = reinterpret_cast<const uint8_t*>(raw);
#pragma unroll
  for (int j = 0; j < E; ++j) {
    if constexpr (DT == kFP16) {
      w[j] = dec_f16(reinterpret_cast<const uint16_t*>(raw)[j]);
    } else if constexpr (w_is_i8(DT)) {
      w[j] = (float)(int8_t)b[j];
    } else if constexpr (w_is_e4m3(DT)) {
      w[j] = dec_e4m3(b[j]);
    } else {  // f4f4, packed along M, low nibble = even column
      w[j] = dec_e2m1((j & 1) ? (b[j >> 1] >> 4) : (b[j >> 1] & 0xF));
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
template <int DT, int NR, int LW>
__global__ void __launch_bounds__(kThreads) gemv_mn_kernel(GemvParams p) {
  using Acc = std::conditional_t<DT == kI8I8, int, float>;
  constexpr int E = LW * 2 / w_bytes_x2<DT>();  // weights per thread
  constexpr int CPC = 32 * E;                   // columns per CTA
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Acc* xs = reinterpret_cast<Acc*>(smem_raw);   // [NR][kchunk]
  const int kc = p.kchunk;
  Acc* red = xs + NR * kc;                      // [NR][CPC]

  const int m0 = blockIdx.x * CPC;
  const int kb = blockIdx.y * kc;
  const int ke = min(p.K, kb + kc);
  const int n0 = blockIdx.z * NR;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  for (int i = tid; i < NR * kc; i += kThreads) {
    const int n = i / kc, k = kb + i % kc;
    Acc v = 0;
    if (n0 + n < p.N && k < ke) {
      if constexpr (DT == kI8I8) {
        v = reinterpret_cast<const int8_t*>(p.X)[(size_t)(n0 + n) * p.K + k];
      } else {
        v = load_x<DT>(p.X, p.xscale, n0 + n, k, p.K);
      }
    }
    xs[i] = v;
  }
  __syncthreads();

  Acc acc[NR][E];
#pragma unroll
  for (int n = 0; n < NR; ++n)
#pragma unroll
    for (int j = 0; j < E; ++j) acc[n][j] = 0;

  const int mc = m0 + lane * E;  // first column owned by this thread
  const size_t row_bytes_x2 = (size_t)p.M * w_bytes_x2<DT>();
  const bool vec = (mc + E <= p.M) && ((row_bytes_x2 / 2) % LW == 0) && (row_bytes_x2 % 2 == 0);
  const uint8_t* wbase = reinterpret_cast<const uint8_t*>(p.W) + (size_t)mc * w_bytes_x2<DT>() / 2;

  if (vec) {
#pragma unroll 4
    for (int k = kb + warp; k < ke; k += kWarps) {
      uint32_t raw[LW / 4];
      const uint8_t* src = wbase + (size_t)k * (row_bytes_x2 / 2);
      if constexpr (LW == 16) {
        const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src));
        raw[0] = v.x; raw[1] = v.y; raw[2] = v.z; raw[3] = v.w;
      } else if constexpr (LW == 8) {
        const uint2 v = __ldcs(reinterpret_cast<const uint2*>(src));
        raw[0] = v.x; raw[1] = v.y;
      } else {
        raw[0] = __ldcs(reinterpret_cast<const unsigned int*>(src));
      }
      const int kl = k - kb;
      if constexpr (DT == kI8I8) {
        const int8_t* b = reinterpret_cast<const int8_t*>(raw);
#pragma unroll
        for (int n = 0; n < NR; ++n) {
          const int xv = xs[n * kc + kl];
#pragma unroll
          for (int j = 0; j < E; ++j) acc[n][j] += xv * (int)b[j];
        }
      } else {
        float w[E];
        decode_w_chunk<DT, E, LW>(raw, w);
#pragma unroll
        for (int n = 0; n < NR; ++n) {
          const float xv = xs[n * kc + kl];
#pragma unroll
          for (int j = 0; j < E; ++j) acc[n][j] = fmaf(xv, w[j], acc[n][j]);
        }
      }
    }
  } else {
    for (int k = kb + warp; k < ke; k += kWarps) {
      const int kl = k - kb;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        const int m = mc + j;
        if (m >= p.M) break;
        if constexpr (DT == kI8I8) {
          const int wv = reinterpret_cast<const int8_t*>(p.W)[(size_t)k * p.M + m];
#pragma unroll
          for (int n = 0; n < NR; ++n) acc[n][j] += xs[n * kc + kl] * wv;
        } else {
          const float wv = load_w_mn<DT>(p.W, k, m, p.M);
#pragma unroll
          for (int n = 0; n < NR; ++n) acc[n][j] = fmaf(xs[n * kc + kl], wv, acc[n][j]);
        }
      }
    }
  }

  // cross-warp reduction in a fixed order (warp 0 first)
  for (int w = 0; w < kWarps; ++w) {
    if (warp == w) {
#pragma unroll
      for (int n = 0; n < NR; ++n)
#pragma unroll
        for (int j = 0; j < E; ++j) {
          Acc* r = &red[n * CPC + lane * E + j];
          *r = (w == 0) ? acc[n][j] : (*r + acc[n][j]);
        }
    }
    __syncthreads();
  }
  finish_tile<Acc>(p, red, n0, NR, m0, CPC);
}

// ---------------------------------------------------------------------------
// [M,K] weights (mxfp4 family): E2M1 packed along K, UE8M0 [M, K/32]
// ---------------------------------------------------------------------------
template <int DT, int NR>
__global__ void __launch_bounds__(kThreads) gemv_km_kernel(GemvParams p) {
  constexpr int RPW = 4;              // output columns per warp
  constexpr int CPC = kWarps * RPW;   // 32 columns per CTA
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw);  // [NR][kchunk]
  const int kc = p.kchunk;
  float* red = xs + NR * kc;                       // [NR][CPC]

  const int m0 = blockIdx.x * CPC;
  const int kb = blockIdx.y * kc;
  const int ke = min(p.K, kb + kc);
  const int n0 = blockIdx.z * NR;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  for (int i = tid; i < NR * kc; i += kThreads) {
    const int n = i / kc, k = kb + i % kc;
    xs[i] = (n0 + n < p.N && k < ke) ? load_x<DT>(p.X, p.xscale, n0 + n, k, p.K) : 0.f;
  }
  __syncthreads();

  float acc[NR][RPW];
#pragma unroll
  for (int n = 0; n < NR; ++n)
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[n][r] = 0.f;

  const int kblocks = (ke - kb) / 32;  // kchunk and K are multiples of 32
  const int kbpr = p.K / 32;           // scale bytes per weight row
  const uint8_t* W = reinterpret_cast<const uint8_t*>(p.W);
  for (int blk = lane; blk < kblocks; blk += 32) {
    const int k = kb + blk * 32;
    uint4 wv[RPW];
    float sc[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int m = m0 + warp * RPW + r;
      if (m < p.M) {
        wv[r] = __ldcs(reinterpret_cast<const uint4*>(W + ((size_t)m * p.K + k) / 2));
        sc[r] = dec_ue8m0(p.wscale[(size_t)m * kbpr + k / 32]);
      } else {
        wv[r] = make_uint4(0, 0, 0, 0);
        sc[r] = 0.f;
      }
    }
    float d[NR][RPW];
#pragma unroll
    for (int n = 0; n < NR; ++n)
#pragma unroll
      for (int r = 0; r < RPW; ++r) d[n][r] = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {        // 4 words x 8 nibbles
#pragma unroll
      for (int h = 0; h < 2; ++h) {      // 4 elements at a time
        float4 xv[NR];
#pragma unroll
        for (int n = 0; n < NR; ++n)
          xv[n] = *reinterpret_cast<const float4*>(&xs[n * kc + blk * 32 + q * 8 + h * 4]);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          const uint32_t word = (&wv[r].x)[q] >> (16 * h);
          const float w0 = dec_e2m1(word), w1 = dec_e2m1(word >> 4);
          const float w2 = dec_e2m1(word >> 8), w3 = dec_e2m1(word >> 12);
#pragma unroll
          for (int n = 0; n < NR; ++n) {
            d[n][r] = fmaf(xv[n].x, w0, d[n][r]);
            d[n][r] = fmaf(xv[n].y, w1, d[n][r]);
            d[n][r] = fmaf(xv[n].z, w2, d[n][r]);
            d[n][r] = fmaf(xv[n].w, w3, d[n][r]);
          }
        }
      }
    }
#pragma unroll
    for (int n = 0; n < NR; ++n)
#pragma unroll
      for (int r = 0; r < RPW; ++r) acc[n][r] = fmaf(d[n][r], sc[r], acc[n][r]);
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
  return 32 * (lw * 2 / bx2);
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
    smem = (size_t)NR * p.kchunk * 4 + (size_t)NR * 32 * 4;
    auto k = gemv_km_kernel<DT, NR>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<grid, kThreads, smem, st>>>(p);
  } else {
    constexpr int LW = pick_lw<DT>(NR);
    constexpr int E = LW * 2 / w_bytes_x2<DT>();
    smem = (size_t)NR * p.kchunk * 4 + (size_t)NR * 32 * E * 4;
    auto k = gemv_mn_kernel<DT, NR, LW>;
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
