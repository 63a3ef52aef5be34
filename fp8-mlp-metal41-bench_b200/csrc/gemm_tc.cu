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
//               for block-scaled kinds it also bulk-copies each stage's
//               pre-packed UE8M0 blocks (sf_pack_kernel) and the MMA issuer
//               moves them to TMEM with tcgen05.cp before each MMA
//   warps 4-7   epilogue: tcgen05.ld TMEM -> registers -> Y, one TMEM lane
//               quadrant (32 output rows) per warp
//
// The grid is persistent (one CTA per SM); output tiles are BM=128 rows of
// Y by BN (128 or 256) columns.  X is always K-major.  W is MN-major for
// the [K,M] dtypes (fp16, i8i8, f8f8: the instruction descriptor's
// "transpose B" bit) and K-major for the [M,K] mxfp4 family.
//
// Kinds per dtype:
//   fp16                 kind::f16       F16 x F16 -> F32
//   i8i8                 kind::i8        S8 x S8 -> S32 (exact)
//   f8f8                 kind::f8f6f4    E4M3 x E4M3 -> F32
//   mxfp4/a4             kind::mxf4      E2M1 x E2M1, UE8M0 per 32 on both
//   f4f4                 kind::mxf4      E2M1 x E2M1 with unit scales (127);
//                                        W [K,M] is first transposed to
//                                        [M,K] into the workspace (the MMA
//                                        needs 4-bit operands K-major)
//   mxfp4/a8, mxfp4/f8   kind::mxf8f6f4  E4M3 x E2M1, UE8M0 per 32; TMA
//                                        unpacks the E2M1 weights into
//                                        8-bit containers (16U4_ALIGN16B)
//
// Every mbarrier wait is bounded (ptx.cuh); on expiry the kernel records
// an error word, lets in-flight TMA copies land, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "formats.cuh"
#include "kernels.h"
#include "ptx.cuh"
#include "tmap.h"
#include "widen.cuh"

namespace mlpg {

namespace {

constexpr int kBM = 128;
constexpr int kThreads = 256;
constexpr int kBarBytes = 512;   // shared memory reserved for the barrier block (Bars) in every kernel
constexpr int kRowBytes = 128;   // bytes of K per operand row per stage (one swizzle row)
constexpr int kSfChunk = 512;    // one 32 x 16-byte scale-factor block (one tcgen05.cp)

// Per-dtype kernel traits.
//   a_bits/b_bits   bits per element as stored in shared memory per K element
//                   (E2M1 for kind::mxf8f6f4 is unpacked to 8 bits by TMA)
//   nsf             UE8M0 scale factors per row per MMA (0 = unscaled kind)
//   x_plane/w_plane the dtype reads an X / W scale plane (else the scale is 1)
template <int DT>
struct Traits;

template <>
struct Traits<kFP16> {
  static constexpr int kind = kKindF16, a_bits = 16, b_bits = 16, nsf = 0;
  static constexpr bool b_mn = true, x_plane = false, w_plane = false, b_unpack4 = false;
  static constexpr uint32_t a_fmt = 0, b_fmt = 0, c_fmt = 1;  // F16, F16 -> F32
};
template <>
struct Traits<kI8I8> {
  static constexpr int kind = kKindI8, a_bits = 8, b_bits = 8, nsf = 0;
  static constexpr bool b_mn = true, x_plane = false, w_plane = false, b_unpack4 = false;
  static constexpr uint32_t a_fmt = 1, b_fmt = 1, c_fmt = 2;  // S8, S8 -> S32
};
template <>
struct Traits<kF8F8> {
  static constexpr int kind = kKindF8F6F4, a_bits = 8, b_bits = 8, nsf = 0;
  static constexpr bool b_mn = true, x_plane = false, w_plane = false, b_unpack4 = false;
  static constexpr uint32_t a_fmt = 0, b_fmt = 0, c_fmt = 1;  // E4M3, E4M3 -> F32
};
template <>
struct Traits<kMX4X4> {
  static constexpr int kind = kKindMxF4, a_bits = 4, b_bits = 4, nsf = 2;
  static constexpr bool b_mn = false, x_plane = true, w_plane = true, b_unpack4 = false;
  static constexpr uint32_t a_fmt = 1, b_fmt = 1, c_fmt = 1;  // E2M1 (mxf4), E2M1
};
template <>
struct Traits<kF4F4> {
  static constexpr int kind = kKindMxF4, a_bits = 4, b_bits = 4, nsf = 2;
  static constexpr bool b_mn = false, x_plane = false, w_plane = false, b_unpack4 = false;
  static constexpr uint32_t a_fmt = 1, b_fmt = 1, c_fmt = 1;
};
template <>
struct Traits<kMX8X4> {
  static constexpr int kind = kKindMxF8F6F4, a_bits = 8, b_bits = 8, nsf = 1;
  static constexpr bool b_mn = false, x_plane = true, w_plane = true, b_unpack4 = true;
  static constexpr uint32_t a_fmt = 0, b_fmt = 5, c_fmt = 1;  // E4M3, E2M1
};
template <>
struct Traits<kF8X4> {
  static constexpr int kind = kKindMxF8F6F4, a_bits = 8, b_bits = 8, nsf = 1;
  static constexpr bool b_mn = false, x_plane = false, w_plane = true, b_unpack4 = true;
  static constexpr uint32_t a_fmt = 0, b_fmt = 5, c_fmt = 1;
};

struct TcParams {
  void* Y;
  const uint8_t* sfa;      // packed X scale blocks (see sf_pack_kernel) or null (scale 1)
  const uint8_t* sfb;      // packed W scale blocks or null (scale 1)
  const int8_t* col_exp;   // per output column: Y *= 2^col_exp (exact), or null
  int N, K, M;
  int tiles_m, tiles_n, num_kb;
  int* dev_err;
  uint32_t* peer[kMaxPeers];   // peer Y bases: every Y store is repeated at the same offset
  int npeers;
  // 1: the epilogue stores Y (and the peers' Y) through the TMA with the maps
  // of EpiMaps (rows of M % 4 == 0 words, Y 16-byte aligned); 0: plain stores
  int y_tma;
  // CTA-pair kernel work items: tiles 0 .. split_from-1 whole, then every
  // later tile as two 256 x BN/2 halves (the last, partial wave spread over
  // twice the pairs); split_from = num_items = the tile count when unsplit
  int split_from, num_items;
};

void set_peers(TcParams& p, const RunArgs& a) {
  p.npeers = a.npeers;
  for (int i = 0; i < kMaxPeers; ++i)
    p.peer[i] = i < a.npeers ? static_cast<uint32_t*>(a.ypeers[i]) : nullptr;
}

constexpr uint32_t pow2_cols(int c) {
  return c <= 32 ? 32u : c <= 64 ? 64u : c <= 128 ? 128u : c <= 256 ? 256u : 512u;
}

template <int DT, int BN, int STAGES>
struct Cfg {
  using T = Traits<DT>;
  static constexpr bool SCALED = T::nsf > 0;
  static constexpr int A_BYTES = kBM * kRowBytes;            // 16 KB
  static constexpr int B_BYTES = BN * kRowBytes;             // 16 / 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // transaction bytes per stage: the 16U4_ALIGN16B load counts the packed
  // 4-bit source bytes (half of what it writes to shared memory)
  static constexpr int STAGE_TX_AB = A_BYTES + (T::b_unpack4 ? B_BYTES / 2 : B_BYTES);
  static constexpr int K_PER_STAGE = kRowBytes * 8 / T::a_bits;  // elements
  static constexpr int MMA_K_BYTES = 32;                     // K bytes per tcgen05.mma
  static constexpr int MMAS_PER_STAGE = kRowBytes / MMA_K_BYTES;  // 4
  static constexpr int KBLK_PER_STAGE = K_PER_STAGE / 32;    // UE8M0 blocks per stage
  // MN-major B: one TMA box is K_PER_STAGE rows x 128 bytes of MN
  static constexpr int B_BOX_MN = kRowBytes * 8 / T::b_bits; // MN elements per box
  static constexpr int B_BOXES = T::b_mn ? BN / B_BOX_MN : 1;
  static constexpr int B_BOX_BYTES = T::b_mn ? K_PER_STAGE * kRowBytes : B_BYTES;
  // descriptor strides
  static constexpr uint32_t B_LBO = T::b_mn ? (uint32_t)B_BOX_BYTES : 16u;
  static constexpr uint32_t B_ADV = T::b_mn ? (uint32_t)(MMA_K_BYTES * 8 / T::b_bits) * kRowBytes
                                            : (uint32_t)MMA_K_BYTES;
  // scale factors: one 32-bit TMEM cell per row holds 4 UE8M0 bytes, which
  // serve 4 MMAs of kind::mxf8f6f4 (one block of 32 each) or 2 of kind::mxf4
  // (two blocks each); the MMA picks its byte with the descriptor's scale-factor
  // id.  Per stage: SF_CELLS 512-byte blocks for A, BN/128 times that for B.
  static constexpr int SF_B_CHUNKS = BN / 128;
  static constexpr int SF_CELLS = SCALED ? MMAS_PER_STAGE * T::nsf / 4 : 0;
  static constexpr int SF_A_BYTES = SF_CELLS * kSfChunk;
  static constexpr int SF_B_BYTES = SF_CELLS * SF_B_CHUNKS * kSfChunk;
  static constexpr int SF_STAGE_BYTES = SF_A_BYTES + SF_B_BYTES;
  static constexpr int SF_OFF = STAGES * STAGE_BYTES;
  static constexpr int SF_CONST_OFF = SF_OFF + STAGES * SF_STAGE_BYTES;   // 512 bytes of 127s
  // TMEM: [0, ACC_BUFS*BN) accumulators; then per stage and cell 4 columns for
  // A and 4*BN/128 for B (one 32-bit column per 32 rows, byte s = block s).
  // Block-scaled 256-wide tiles keep one accumulator: two would fill all 512
  // columns and leave none for the scale cells (the epilogue then drains the
  // accumulator before the next tile's first MMA).
  static constexpr int ACC_BUFS = (SCALED && BN == 256) ? 1 : 2;
  static constexpr int ACC_COLS = BN;
  static constexpr int SF_COL0 = ACC_BUFS * BN;
  static constexpr int SF_COLS_A = 4, SF_COLS_B = 4 * SF_B_CHUNKS;
  static constexpr int SF_COLS_STAGE = SF_CELLS * (SF_COLS_A + SF_COLS_B);
  static constexpr uint32_t TMEM_COLS = pow2_cols(ACC_BUFS * BN + STAGES * SF_COLS_STAGE);
  static constexpr int BAR_OFF = SF_CONST_OFF + (SCALED ? kSfChunk : 0);
  static constexpr int SMEM_BYTES = BAR_OFF + kBarBytes + 1024;    // + barriers + alignment slack
  // TMA-store epilogue: 4 KB staging buffers per epilogue warp, two where the
  // shared-memory budget allows (a chunk's store overlaps the next chunk's
  // staging), else one
  static constexpr int EPI_OFF = (BAR_OFF + kBarBytes + 1023) / 1024 * 1024;
  static constexpr int EPI_BUFS = EPI_OFF + 4 * 2 * 4096 + 1024 <= 232448 ? 2 : 1;
  static constexpr int SMEM_EPI = EPI_OFF + 4 * EPI_BUFS * 4096 + 1024;
  static constexpr uint32_t IDESC =
      SCALED ? ((T::a_fmt << 7) | (T::b_fmt << 10) | ((uint32_t)(BN >> 3) << 17) | (1u << 23) |
                ((uint32_t)(kBM >> 4) << 24))
             : ((T::c_fmt << 4) | (T::a_fmt << 7) | (T::b_fmt << 10) |
                ((T::b_mn ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                ((uint32_t)(kBM >> 4) << 24));
  static_assert(BN % 16 == 0 && BN <= 256, "UMMA N");
  static_assert(!T::b_mn || BN % B_BOX_MN == 0, "MN-major B tile must be whole swizzle atoms");
  static_assert(ACC_BUFS * BN + STAGES * SF_COLS_STAGE <= 512, "TMEM budget");
  static_assert(SMEM_EPI <= 232448, "shared memory budget");
};

// Tensor maps of the epilogue's TMA stores: this GPU's Y and the peers' Y
// blocks (fused all-gather), each [N, M] of 32-bit words from its base
// pointer, 32 x 32 boxes, 128-byte swizzle.
struct EpiMaps {
  CUtensorMap y;
  CUtensorMap m[kMaxPeers];
};

struct Bars {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
  uint64_t sf_ready[8];   // block-scaled kinds: a stage's scale cells are in TMEM
  uint64_t sf_free[8];    // block-scaled pair tiles with fewer TMEM scale slots than stages
};
static_assert(sizeof(Bars) <= kBarBytes, "barrier block");

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int& tm, int& tn) {
  tm = tile % tiles_m;
  tn = tile / tiles_m;
}

// Work item i of the CTA-pair kernel: its tile and, for a half tile, which
// half of the tile's columns (-1: the whole tile).
__device__ __forceinline__ void item_coords(int i, const TcParams& p, int& tm, int& tn, int& half) {
  int t = i;
  half = -1;
  if (i >= p.split_from) {
    const int j = i - p.split_from;
    t = p.split_from + (j >> 1);
    half = j & 1;
  }
  tile_coords(t, p.tiles_m, tm, tn);
}

// Scale-factor packing pre-pass.  For every 128-row tile t of an operand,
// every K stage st and every cell g of the stage (4 k-blocks), one 512-byte
// block: byte (16*r0 + 4*j + s) = UE8M0 scale of row 128*t + r0 + 32*j for
// k-block st*nb + 4*g + s (127 = 1.0 outside the matrix).  That is the source
// layout of tcgen05.cp.32x128b.warpx4: row r0's 16 bytes land in TMEM lane r0
// of every lane quadrant, 32-bit column j, where the block-scaled MMA reads the
// scales of row r0 + 32*j, byte s selected by the descriptor's scale-factor id.
// The producer then fetches each stage's blocks with one 1-D bulk copy per
// operand.
struct SfPackJob {
  const uint8_t* plane;   // [rows, kbpr]
  uint8_t* out;           // [tiles][stages][cells][512]
  int rows, tiles;        // tiles: packed 128-row blocks (chunks) in all
  int tile_rows;          // operand rows per MMA tile (128, 192 or 256)
  int chunks;             // 128-row chunks per MMA tile: ceil(tile_rows / 128)
};

__global__ void __launch_bounds__(256) sf_pack_kernel(SfPackJob ja, SfPackJob jb, int kbpr, int stages, int nb,
                                                      int cells) {
  const SfPackJob& job = blockIdx.y == 0 ? ja : jb;      // y = 0: X plane, 1: W plane
  if (job.plane == nullptr) return;
  const int tid = blockIdx.x * 256 + threadIdx.x;       // one thread per (t, st, g, r0)
  const int r0 = tid & 31;
  const int g = (tid >> 5) % cells;
  const int rest = (tid >> 5) / cells;
  const int st = rest % stages, t = rest / stages;
  if (t >= job.tiles) return;
  const uint8_t* plane = job.plane;
  const int rows = job.rows;
  uint8_t* out = job.out;
  // packed block t is chunk c of MMA tile t_outer: rows t_outer * tile_rows + 128 c + ...
  const int t_outer = t / job.chunks, c = t % job.chunks;
  const int tile_rows = job.tile_rows;
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int row_in = c * 128 + r0 + 32 * j;   // row within the MMA tile
    const int row = t_outer * tile_rows + row_in;
    uint32_t v = 0;
    for (int q = 0; q < 4; ++q) {
      const int kblk = st * nb + 4 * g + q;
      const uint32_t sc =
          (row_in < tile_rows && row < rows && kblk < kbpr) ? plane[(size_t)row * kbpr + kblk] : 127u;
      v |= sc << (8 * q);
    }
    w[j] = v;
  }
  *reinterpret_cast<uint4*>(out + ((size_t)((t * stages + st) * cells + g)) * 512 + r0 * 16) =
      make_uint4(w[0], w[1], w[2], w[3]);
}

// Epilogue of one TMEM lane quadrant (32 output rows): NCH chunks of 32
// accumulator columns.  The TMEM load of chunk c+1 is in flight while chunk c
// is stored, and `release` runs as soon as the last load has completed, so the
// next tile's MMAs may overwrite the accumulator while the last chunk is still
// being stored.
//
// With peers (the fused all-gather), each chunk is stored again at the same
// offset in every peer's Y over NVLink; the stores are plain posted writes,
// made visible to the peers by the kernel's end.  Over NVLink every store
// instruction should write whole 128-byte lines, not 16 bytes in each of 32
// rows, so the warp first rearranges the chunk with shuffles (peer_layout).
__device__ __forceinline__ void store_chunk(uint32_t* yrow, const uint32_t (&r)[32], int cb, int M, bool vec_ok) {
  if (vec_ok && cb + 32 <= M) {
    uint4* dst = reinterpret_cast<uint4*>(yrow + cb);
#pragma unroll
    for (int v = 0; v < 8; ++v) dst[v] = make_uint4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
  } else {
#pragma unroll
    for (int v = 0; v < 32; ++v)
      if (cb + v < M) yrow[cb + v] = r[v];
  }
}

// A 32 x 32 chunk held one row per lane (r[v] = column v of row `lane`) is
// rearranged so that register group j of lane L holds columns 4(L>>2) ..
// 4(L>>2)+3 of row 4j + (L&3): three butterfly stages, each swapping one bit
// of the register group index (k) with lane bit k+2.  Afterwards each group
// of 8 lanes with the same L&3 covers one row's 128 bytes.
__device__ __forceinline__ void peer_layout(uint32_t (&r)[32], int lane) {
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const int m = 1 << (k + 2);
    const bool hi = (lane & m) != 0;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      if (g & (1 << k)) continue;
      const int gb = g | (1 << k);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t send = hi ? r[4 * g + e] : r[4 * gb + e];
        const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, m);
        if (hi) r[4 * g + e] = recv;
        else r[4 * gb + e] = recv;
      }
    }
  }
}

// Peer stores of one chunk (whole warp): rows row0 .. row0+31 of Y, columns
// cb .. cb+31, rows at or past N skipped.
__device__ __forceinline__ void store_peers(uint32_t (&r)[32], const TcParams& p, int row0, int cb, int M,
                                            bool vec_ok, bool row_ok) {
  const int lane = (int)(threadIdx.x & 31u);
  if (!vec_ok) {   // rows of M % 4 floats are not 16-byte aligned: one lane per row
    if (!row_ok) return;
#pragma unroll
    for (int i = 0; i < kMaxPeers; ++i)
      if (i < p.npeers) store_chunk(p.peer[i] + (size_t)(row0 + lane) * M, r, cb, M, false);
    return;
  }
  peer_layout(r, lane);
  const int col = cb + 4 * (lane >> 2);
  if (col >= M) return;   // M % 4 == 0: a group is all in or all out
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int row = row0 + ((j << 2) | (lane & 3));
    if (row >= p.N) continue;
    const uint4 v = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
    const size_t off = (size_t)row * M + col;
#pragma unroll
    for (int i = 0; i < kMaxPeers; ++i)
      if (i < p.npeers) *reinterpret_cast<uint4*>(p.peer[i] + off) = v;
  }
}

// Peer stores of one chunk through the TMA (whole warp): the chunk goes to
// this warp's 4 KB staging buffer (`epi`, 1024-byte aligned) with the 128-byte
// swizzle, which keeps the 32 row writes free of bank conflicts, and lane 0
// stores the 32 x 32 box to every peer's map at (cb, row0).  The next chunk
// waits until the TMA has read the buffer.
__device__ __forceinline__ void store_peers_tma(const uint32_t (&r)[32], unsigned char* epi, const EpiMaps* pm,
                                                int npeers, int row0, int cb, int N, int M) {
  const int lane = (int)(threadIdx.x & 31u);
  const uint32_t base = smem_u32(epi);
#pragma unroll
  for (int v = 0; v < 8; ++v) {
    const uint32_t a = base + (uint32_t)lane * 128u + (uint32_t)((v ^ (lane & 7)) << 4);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(r[4 * v]), "r"(r[4 * v + 1]),
                 "r"(r[4 * v + 2]), "r"(r[4 * v + 3])
                 : "memory");
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (row0 < N && cb < M) {
      for (int i = 0; i < npeers; ++i) tma_store_2d(&pm->m[i], base, cb, row0);
      bulk_commit_group();
    }
    bulk_wait_read_all();
  }
  __syncwarp();
}

// f32 results of one 32-column chunk times 2^e per column (exact powers of
// two; the A16 mxfp4 path's per-column exponent offsets).  The chunk's 32
// exponents come in two 16-byte loads (the same for every lane); nothing is
// done when all are zero, the usual case.
__device__ __forceinline__ void apply_col_exp(uint32_t (&r)[32], const int8_t* col_exp, int cb, int M) {
  uint32_t e4[8];
  if (cb + 32 <= M) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(col_exp + cb));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(col_exp + cb + 16));
    e4[0] = a.x, e4[1] = a.y, e4[2] = a.z, e4[3] = a.w, e4[4] = b.x, e4[5] = b.y, e4[6] = b.z, e4[7] = b.w;
  } else {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      uint32_t x = 0;
      for (int i = 0; i < 4; ++i)
        if (cb + 4 * w + i < M) x |= (uint32_t)(uint8_t)col_exp[cb + 4 * w + i] << (8 * i);
      e4[w] = x;
    }
  }
  if ((e4[0] | e4[1] | e4[2] | e4[3] | e4[4] | e4[5] | e4[6] | e4[7]) != 0u) {
#pragma unroll
    for (int v = 0; v < 32; ++v) {
      const int e = (int)(int8_t)(e4[v >> 2] >> (8 * (v & 3)));
      if (e) r[v] = __float_as_uint(__uint_as_float(r[v]) * __int_as_float((e + 127) << 23));
    }
  }
}

template <int NCH, typename Release>
__device__ __forceinline__ void drain_quadrant(uint32_t taddr0, uint32_t* yrow, int col0, int M, bool row_ok,
                                               const int8_t* col_exp, const TcParams& p, int row0,
                                               Release release, unsigned char* epi = nullptr,
                                               const EpiMaps* pm = nullptr) {
  const bool vec_ok = (M % 4) == 0;
  // this lane's row: column exponents (if any), then the local store
  auto store_row = [&](uint32_t (&r)[32], int cb) {
    if (col_exp) apply_col_exp(r, col_exp, cb, M);
    store_chunk(yrow, r, cb, M, vec_ok);
  };
  auto store = [&](uint32_t (&r)[32], int c) {
    const int cb = col0 + c * 32;
    if (p.npeers) {   // the whole warp takes part in the peer stores
      if (row_ok) store_row(r, cb);
      if (epi && vec_ok) store_peers_tma(r, epi, pm, p.npeers, row0, cb, p.N, M);
      else store_peers(r, p, row0, cb, M, vec_ok, row_ok);
      return;
    }
    if (!row_ok) return;
    store_row(r, cb);
  };
  uint32_t ra[32], rb[32];
  tmem_ld_32x32b_x32(taddr0, ra);
#pragma unroll 1
  for (int c = 0; c < NCH; c += 2) {
    tmem_ld_wait();                                            // chunk c in ra
    if (c + 1 < NCH) tmem_ld_32x32b_x32(taddr0 + (uint32_t)((c + 1) * 32), rb);
    else release();                                            // an odd last chunk
    store(ra, c);
    if (c + 1 >= NCH) break;
    tmem_ld_wait();                                            // chunk c + 1 in rb
    if (c + 2 < NCH) tmem_ld_32x32b_x32(taddr0 + (uint32_t)((c + 2) * 32), ra);
    else release();
    store(rb, c + 1);
  }
}

// Epilogue of one 32-row TMEM lane quadrant through the TMA (whole warp).
// Each 32 x 32 chunk goes TMEM -> registers (tcgen05.ld), gets its column
// exponents (if any), and is written into one of this warp's NBUF 4 KB
// staging buffers (`epi`, 1024-byte aligned) with the 128-byte swizzle, so
// the 32 row writes are free of bank conflicts; lane 0 then stores the
// 32 x 32 box to this GPU's Y and to every peer's Y with one
// cp.async.bulk.tensor each (rows past N and columns past M are clipped by
// the TMA).  Compared with one 16-byte store per lane into 32 different rows,
// the TMA writes whole 128-byte lines and leaves the SM's load/store path to
// the operand stream.  `nst` counts this warp's stored chunks across tiles:
// buffer nst % NBUF is rewritten only after the TMA has read it, i.e. once at
// most NBUF - 1 newer store groups are pending.  Chunks with nothing to store
// (past M, or a quadrant past N) write no buffer and commit no group; stored
// chunks are a prefix of the tile's chunks.  `release` frees the accumulator
// once the last chunk is in registers.
template <int NCH, int NBUF, typename Release>
__device__ __forceinline__ void drain_quadrant_tma(uint32_t taddr0, int col0, int row0, const TcParams& p,
                                                   Release release, unsigned char* epi, const EpiMaps* em,
                                                   int& nst) {
  static_assert(NBUF >= 1 && NBUF <= 2, "one or two staging buffers");
  const int lane = (int)(threadIdx.x & 31u);
  auto put = [&](uint32_t (&r)[32], int c) {
    const int cb = col0 + c * 32;
    if (row0 >= p.N || cb >= p.M) return;
    if (p.col_exp) apply_col_exp(r, p.col_exp, cb, p.M);
    const uint32_t base = smem_u32(epi) + (uint32_t)((nst % NBUF) * 4096);
    if (lane == 0) bulk_wait_read<NBUF - 1>();   // the buffer's previous store has read it
    __syncwarp();
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      const uint32_t a = base + (uint32_t)lane * 128u + (uint32_t)((v ^ (lane & 7)) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(r[4 * v]), "r"(r[4 * v + 1]),
                   "r"(r[4 * v + 2]), "r"(r[4 * v + 3])
                   : "memory");
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(&em->y, base, cb, row0);
      for (int i = 0; i < p.npeers; ++i) tma_store_2d(&em->m[i], base, cb, row0);
      bulk_commit_group();
    }
    ++nst;
  };
  // TMEM loads in groups of two chunks (two 32-column loads in flight per wait),
  // double-buffered: group g + 1 loads while group g is staged and stored; an
  // odd chunk count ends with a group of one
  constexpr int NG = (NCH + 1) / 2;
  uint32_t ra0[32], ra1[32], rb0[32], rb1[32];
  auto load_group = [&](int g, uint32_t (&x0)[32], uint32_t (&x1)[32]) {
    tmem_ld_32x32b_x32(taddr0 + (uint32_t)((2 * g) * 32), x0);
    if (2 * g + 1 < NCH) tmem_ld_32x32b_x32(taddr0 + (uint32_t)((2 * g + 1) * 32), x1);
  };
  load_group(0, ra0, ra1);
#pragma unroll 1
  for (int g = 0; g < NG; g += 2) {
    tmem_ld_wait();                                            // group g in ra
    if (g + 1 < NG) load_group(g + 1, rb0, rb1);
    else release();
    put(ra0, 2 * g);
    if (2 * g + 1 < NCH) put(ra1, 2 * g + 1);
    if (g + 1 >= NG) break;
    tmem_ld_wait();                                            // group g + 1 in rb
    if (g + 2 < NG) load_group(g + 2, ra0, ra1);
    else release();
    put(rb0, 2 * g + 2);
    if (2 * g + 3 < NCH) put(rb1, 2 * g + 3);
  }
}

template <int DT, int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ EpiMaps em, TcParams p) {
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
    if constexpr (C::SCALED)
      for (int st = 0; st < STAGES; ++st) mbar_init(&bars->sf_ready[st], 1);
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  if constexpr (C::SCALED) {
    // a block of unit scales (127) for operands without a scale plane
    if (warp == 2) {
      *reinterpret_cast<uint4*>(smem + C::SF_CONST_OFF + lane * 16) =
          make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
      fence_proxy_async_smem();
    }
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
    const uint32_t tx = C::STAGE_TX_AB + (p.sfa ? C::SF_A_BYTES : 0) + (p.sfb ? C::SF_B_BYTES : 0);
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, tm, tn);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&bars->empty[stage], phase ^ 1u, ctl, 0x100 + stage)) { ok = false; break; }
        unsigned char* a_dst = smem + stage * C::STAGE_BYTES;
        unsigned char* b_dst = a_dst + C::A_BYTES;
        mbar_arrive_expect_tx(&bars->full[stage], tx);
        if constexpr (C::SCALED) {
          unsigned char* sf = smem + C::SF_OFF + stage * C::SF_STAGE_BYTES;
          if (p.sfa)
            bulk_load(sf, p.sfa + (size_t)(tm * p.num_kb + kb) * C::SF_A_BYTES, C::SF_A_BYTES, &bars->full[stage]);
          if (p.sfb) {
#pragma unroll
            for (int c = 0; c < C::SF_B_CHUNKS; ++c)
              bulk_load(sf + C::SF_A_BYTES + c * C::SF_A_BYTES,
                        p.sfb + (size_t)((tn * C::SF_B_CHUNKS + c) * p.num_kb + kb) * C::SF_A_BYTES,
                        C::SF_A_BYTES, &bars->full[stage]);
          }
        }
        // A tile: x in elements of the map (bytes for 8/4-bit maps)
        tma_load_2d(a_dst, &tmA, &bars->full[stage], kb * (T::a_bits == 16 ? C::K_PER_STAGE : kRowBytes),
                    tm * kBM);
        if constexpr (T::b_mn) {
#pragma unroll
          for (int j = 0; j < C::B_BOXES; ++j)
            tma_load_2d(b_dst + j * C::B_BOX_BYTES, &tmB, &bars->full[stage],
                        tn * BN + j * C::B_BOX_MN, kb * C::K_PER_STAGE);
        } else {
          // K-major B; x counts 4-bit elements for the unpacking map, bytes otherwise
          tma_load_2d(b_dst, &tmB, &bars->full[stage], T::b_unpack4 ? kb * C::K_PER_STAGE : kb * kRowBytes,
                      tn * BN);
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
  } else if (C::SCALED && warp == 3 && lane == 0) {
    // --------------------- scale-cell copier (block-scaled kinds) ---------------
    // A stage's scale blocks go to TMEM with tcgen05.cp from this thread, which
    // commits them to the stage's sf_ready barrier; the MMA issuer waits on that
    // barrier in place of `full`.  With the copies in the MMA thread's own loop
    // (right before each stage's MMAs) the block-scaled tiles measured 7-14 %
    // slower: that single thread paces these kernels.
    // (an operand without a scale plane has unit cells, which the MMA issuer
    // copies into every slot once; with no plane at all this thread has no work)
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    const bool work = p.sfa || p.sfb;
    const uint32_t smem_base = smem_u32(smem);
    for (int tile = blockIdx.x; work && tile < num_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&bars->full[stage], phase, ctl, 0x500 + stage)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sf_smem = smem_base + C::SF_OFF + stage * C::SF_STAGE_BYTES;
        const uint32_t sf_tmem = tmem_base + (uint32_t)(C::SF_COL0 + stage * C::SF_COLS_STAGE);
#pragma unroll
        for (int g = 0; g < C::SF_CELLS; ++g) {
          const uint32_t sfa_t = sf_tmem + g * (C::SF_COLS_A + C::SF_COLS_B);
          if (p.sfa) tc_cp_32x128b_warpx4(sfa_t, sdesc_plain(sf_smem + g * kSfChunk, 0, 128));
          if (p.sfb) {
#pragma unroll
            for (int c = 0; c < C::SF_B_CHUNKS; ++c)
              tc_cp_32x128b_warpx4(sfa_t + C::SF_COLS_A + 4 * c,
                                   sdesc_plain(sf_smem + C::SF_A_BYTES + (c * C::SF_CELLS + g) * kSfChunk, 0, 128));
          }
        }
        tc_commit(&bars->sf_ready[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------ MMA issuer --------------------------------
    uint32_t stage = 0, phase = 0;
    int local = 0;
    bool ok = true;
    const uint32_t smem_base = smem_u32(smem);
    if constexpr (C::SCALED) {
      // unit scale cells (the block of 127s) for an operand without a scale
      // plane go into every ring slot once; this thread's MMAs follow them in
      // issue order
      const uint32_t sf_const = smem_base + C::SF_CONST_OFF;
      for (int st = 0; st < STAGES; ++st) {
        const uint32_t sf_tmem = tmem_base + (uint32_t)(C::SF_COL0 + st * C::SF_COLS_STAGE);
#pragma unroll
        for (int g = 0; g < C::SF_CELLS; ++g) {
          const uint32_t sfa_t = sf_tmem + g * (C::SF_COLS_A + C::SF_COLS_B);
          if (!p.sfa) tc_cp_32x128b_warpx4(sfa_t, sdesc_plain(sf_const, 0, 128));
          if (!p.sfb) {
#pragma unroll
            for (int c = 0; c < C::SF_B_CHUNKS; ++c)
              tc_cp_32x128b_warpx4(sfa_t + C::SF_COLS_A + 4 * c, sdesc_plain(sf_const, 0, 128));
          }
        }
      }
    }
    const bool via_copier = C::SCALED && (p.sfa || p.sfb);
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
      const int buf = C::ACC_BUFS == 2 ? (local & 1) : 0;
      const uint32_t acc_par = C::ACC_BUFS == 2 ? (uint32_t)(local >> 1) & 1u : (uint32_t)local & 1u;
      if (!mbar_wait(&bars->acc_empty[buf], acc_par ^ 1u, ctl, 0x200 + buf)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(buf * C::ACC_COLS);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        // block-scaled kinds: the copier has also put the stage's scale cells in TMEM
        uint64_t* ready = via_copier ? &bars->sf_ready[stage] : &bars->full[stage];
        if (!mbar_wait(ready, phase, ctl, 0x300 + stage)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_base + stage * C::STAGE_BYTES;
        const uint32_t b_addr = a_addr + C::A_BYTES;
        if constexpr (C::SCALED) {
          const uint32_t sf_tmem = tmem_base + (uint32_t)(C::SF_COL0 + stage * C::SF_COLS_STAGE);
#pragma unroll
          for (int kk = 0; kk < C::MMAS_PER_STAGE; ++kk) {
            constexpr int per_cell = 4 / T::nsf;   // MMAs served by one cell
            const int g = kk / per_cell;
            const uint32_t sfid = (uint32_t)((kk % per_cell) * T::nsf);   // first byte of this MMA's blocks
            const uint32_t sfa_t = sf_tmem + g * (C::SF_COLS_A + C::SF_COLS_B);
            const uint32_t sfb_t = sfa_t + C::SF_COLS_A;
            const uint32_t idesc = C::IDESC | (sfid << 4) | (sfid << 29);   // B and A scale-factor ids
            const uint64_t adesc = sdesc_sw128(a_addr + kk * C::MMA_K_BYTES, 16, 1024);
            const uint64_t bdesc = sdesc_sw128(b_addr + kk * C::B_ADV, C::B_LBO, 1024);
            tc_mma_bs<T::kind>(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u, sfa_t, sfb_t);
          }
        } else {
#pragma unroll
          for (int kk = 0; kk < C::MMAS_PER_STAGE; ++kk) {
            const uint64_t adesc = sdesc_sw128(a_addr + kk * C::MMA_K_BYTES, 16, 1024);
            const uint64_t bdesc = sdesc_sw128(b_addr + kk * C::B_ADV, C::B_LBO, 1024);
            tc_mma<T::kind>(d_tmem, adesc, bdesc, C::IDESC, (kb | kk) != 0 ? 1u : 0u);
          }
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
    int nst = 0;   // chunks this warp has stored through the TMA
    unsigned char* epi = smem + C::EPI_OFF + q * C::EPI_BUFS * 4096;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, tm, tn);
      const int buf = C::ACC_BUFS == 2 ? (local & 1) : 0;
      const uint32_t acc_par = C::ACC_BUFS == 2 ? (uint32_t)(local >> 1) & 1u : (uint32_t)local & 1u;
      const bool got = mbar_wait(&bars->acc_full[buf], acc_par, ctl, 0x400 + buf);
      if (!__all_sync(0xffffffffu, got)) break;   // the warp leaves together
      __syncwarp();                               // tcgen05.ld is .sync.aligned
      tc_fence_after();
      const int row = tm * kBM + q * 32 + lane;
      const int col0 = tn * BN;
      const bool row_ok = row < p.N;
      uint32_t* yrow = reinterpret_cast<uint32_t*>(p.Y) + (size_t)row * p.M;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * C::ACC_COLS);
      auto release = [&] {
        tc_fence_before();
        mbar_arrive(&bars->acc_empty[buf]);
      };
      if (p.y_tma)
        drain_quadrant_tma<BN / 32, C::EPI_BUFS>(taddr, col0, row - lane, p, release, epi, &em, nst);
      else
        drain_quadrant<BN / 32>(taddr, yrow, col0, p.M, row_ok, p.col_exp, p, row - lane, release);
    }
    // TMA stores still in flight complete before the CTA ends
    if (p.y_tma && lane == 0) bulk_wait_all();
    __syncwarp();
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
// f4f4: W [K,M] packed along M -> Wt [M,K] packed along K (the 4-bit MMA
// operands must be K-major).  One CTA transposes a 64 (K) x 256 (M) nibble
// tile through shared memory; each thread assembles 32 nibbles of one output
// row (16 bytes) and stores them with one 16-byte store.
// ----------------------------------------------------------------------------
constexpr int kTrK = 64, kTrM = 256;

__global__ void __launch_bounds__(256) transpose_fp4_kernel(const uint8_t* __restrict__ W,
                                                            uint8_t* __restrict__ Wt, int K, int M) {
  __shared__ __align__(16) uint8_t tile[kTrK][kTrM / 2];   // 64 rows x 128 bytes
  const int k0 = blockIdx.y * kTrK, m0 = blockIdx.x * kTrM;
  const int t = threadIdx.x;
  const size_t row_bytes = (size_t)M / 2;                    // M is even
  // load: 64 rows x 8 uint4
  for (int i = t; i < kTrK * 8; i += 256) {
    const int r = i >> 3, c = i & 7;
    const int k = k0 + r;
    const int mb = m0 / 2 + c * 16;                          // byte column
    uint4 v = make_uint4(0, 0, 0, 0);
    if (k < K) {
      const uint8_t* src = W + (size_t)k * row_bytes + mb;
      if (mb + 16 <= (int)row_bytes && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        v = __ldg(reinterpret_cast<const uint4*>(src));
      } else {
        uint8_t b[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) b[j] = (mb + j < (int)row_bytes) ? src[j] : 0;
        v = *reinterpret_cast<uint4*>(b);
      }
    }
    *reinterpret_cast<uint4*>(&tile[r][c * 16]) = v;
  }
  __syncthreads();
  // store: 256 output rows x 2 halves of 32 nibbles
  for (int i = t; i < kTrM * 2; i += 256) {
    const int mr = i >> 1, h = i & 1;
    const int m = m0 + mr;
    const int kk0 = h * 32;
    if (m >= M || k0 + kk0 >= K) continue;
    const int byte = mr >> 1, hi = mr & 1;
    uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const uint32_t nib = (tile[kk0 + j][byte] >> (hi * 4)) & 0xFu;
      o[j >> 3] |= nib << ((j & 7) * 4);
    }
    uint8_t* dst = Wt + (size_t)m * (K / 2) + (k0 + kk0) / 2;
    if (k0 + kk0 + 32 <= K) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
      const uint8_t* b = reinterpret_cast<const uint8_t*>(o);
      for (int j = 0; j < (K - k0 - kk0) / 2; ++j) dst[j] = b[j];
    }
  }
}

// ----------------------------------------------------------------------------
// 2-CTA variant (cta_group::2): a cluster of two CTAs on two SMs computes a
// 256 x BN tile.  Each CTA loads its own 128 rows of X and its own BN/2
// columns of W (halving the operand stream per SM against the 1-CTA 128 x BN
// tile), the pair's leader issues tcgen05.mma.cta_group::2 (M = 256) over
// both CTAs' shared memory, and each CTA's TMEM holds its 128 rows of the
// accumulator.  Completion of both CTAs' TMA loads is counted on the
// leader's "full" barrier; the leader's tcgen05.commit multicasts to the
// "empty" / "acc_full" barriers of both CTAs; both epilogues release the
// accumulator on the leader's "acc_empty".  No TMA load uses multicast.
// ----------------------------------------------------------------------------
template <int DT, int BN, int STAGES>
struct Cfg2 {
  using T = Traits<DT>;
  static constexpr int BH = BN / 2;                          // W columns per CTA
  static constexpr int A_BYTES = kBM * kRowBytes;
  static constexpr int B_BYTES = BH * kRowBytes;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // 4-bit W unpacked into 8-bit containers by TMA (16U4_ALIGN16B); those loads
  // count the packed source bytes, half of what they write
  static constexpr bool B_UNPACK = T::b_unpack4;
  static constexpr int STAGE_TX = A_BYTES + (B_UNPACK ? B_BYTES / 2 : B_BYTES);
  // block-scaled kinds: per stage SF_CELLS 512-byte scale blocks for this CTA's
  // 128 rows of A and for all BN columns of B (each CTA's TMEM holds the scales
  // of every column the pair's MMA multiplies its rows with), as in Cfg
  static constexpr bool SCALED = T::nsf > 0;
  static constexpr int SF_CELLS = SCALED ? (kRowBytes / 32) * T::nsf / 4 : 0;
  static constexpr int SF_B_CHUNKS = (BN + 127) / 128;   // 128-row scale chunks of the B tile
  static constexpr int SF_A_BYTES = SF_CELLS * kSfChunk;
  static constexpr int SF_B_BYTES = SF_CELLS * SF_B_CHUNKS * kSfChunk;
  static constexpr int SF_STAGE_BYTES = SF_A_BYTES + SF_B_BYTES;
  static constexpr int SF_COLS_A = 4, SF_COLS_B = 4 * SF_B_CHUNKS;
  static constexpr int SF_COLS_STAGE = SF_CELLS * (SF_COLS_A + SF_COLS_B);
  // TMEM scale slots: one per ring stage where they fit beside two
  // accumulators in the 512 TMEM columns (a 256x192 scaled tile: 384 + 5 x 24);
  // else at least two, each reused once the MMAs of the stage that held it have
  // completed (sf_free: a 256x224 mxf4 tile, 448 + 2 x 24).  256-wide scaled
  // tiles, whose two accumulators would leave no column for the scales, keep a
  // slot per stage and one accumulator.
  static constexpr int SF_FIT = SCALED ? (512 - 2 * BN) / SF_COLS_STAGE : 0;
  static constexpr int SF_SLOTS = !SCALED ? 0 : (SF_FIT >= STAGES ? STAGES : (SF_FIT >= 2 ? SF_FIT : STAGES));
  static constexpr int ACC_BUFS = (!SCALED || 2 * BN + SF_SLOTS * SF_COLS_STAGE <= 512) ? 2 : 1;
  static constexpr int K_PER_STAGE = kRowBytes * 8 / T::a_bits;
  static constexpr int MMA_K_BYTES = 32;
  static constexpr int MMAS_PER_STAGE = kRowBytes / MMA_K_BYTES;
  static constexpr int B_BOX_MN = kRowBytes * 8 / T::b_bits;
  static constexpr int B_BOXES = T::b_mn ? BH / B_BOX_MN : 1;
  static constexpr int B_BOX_BYTES = T::b_mn ? K_PER_STAGE * kRowBytes : B_BYTES;
  static constexpr uint32_t B_LBO = T::b_mn ? (uint32_t)B_BOX_BYTES : 16u;
  static constexpr uint32_t B_ADV = T::b_mn ? (uint32_t)(MMA_K_BYTES * 8 / T::b_bits) * kRowBytes
                                            : (uint32_t)MMA_K_BYTES;
  static constexpr int SF_COL0 = ACC_BUFS * BN;
  static constexpr uint32_t TMEM_COLS = pow2_cols(ACC_BUFS * BN + SF_SLOTS * SF_COLS_STAGE);
  static constexpr int SF_OFF = STAGES * STAGE_BYTES;
  static constexpr int SF_CONST_OFF = SF_OFF + STAGES * SF_STAGE_BYTES;   // 512 bytes of 127s
  static constexpr int BAR_OFF = SF_CONST_OFF + (SCALED ? kSfChunk : 0);
  // TMA-store epilogue: 4 KB staging buffers per epilogue warp, two where the
  // shared-memory budget allows, else one; none (plain stores) if even one
  // does not fit beside the ring
  static constexpr int EPI_OFF = (BAR_OFF + kBarBytes + 1023) / 1024 * 1024;
  static constexpr int EPI_BUFS = EPI_OFF + 4 * 2 * 4096 + 1024 <= 232448   ? 2
                                  : EPI_OFF + 4 * 1 * 4096 + 1024 <= 232448 ? 1
                                                                            : 0;
  static constexpr bool EPI_TMA = EPI_BUFS > 0;
  static constexpr int SMEM_BYTES = (EPI_TMA ? EPI_OFF + 4 * EPI_BUFS * 4096 : BAR_OFF + kBarBytes) + 1024;
  static constexpr int SMEM_BASE = BAR_OFF + kBarBytes + 1024;   // launches with plain epilogue stores
  static constexpr uint32_t IDESC =
      SCALED ? ((T::a_fmt << 7) | (T::b_fmt << 10) | ((uint32_t)(BN >> 3) << 17) | (1u << 23) |
                ((uint32_t)(256 >> 4) << 24))
             : ((T::c_fmt << 4) | (T::a_fmt << 7) | (T::b_fmt << 10) | ((T::b_mn ? 1u : 0u) << 16) |
                ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24));
  // half tiles (256 x BN/2): unscaled kinds without 4-bit unpacking
  static constexpr bool HALVES = !SCALED && !B_UNPACK && (!T::b_mn || (BH / 2) % B_BOX_MN == 0);
  static constexpr int STAGE_TX_H = A_BYTES + B_BYTES / 2;
  static constexpr uint32_t IDESC_H = (IDESC & ~(0x3Fu << 17)) | ((uint32_t)(BN / 2 >> 3) << 17);
  static_assert(ACC_BUFS * BN + SF_SLOTS * SF_COLS_STAGE <= 512, "TMEM budget");
  static_assert(SF_SLOTS <= 8, "sf_free barriers");
  static_assert(!T::b_mn || BH % B_BOX_MN == 0, "W half-tile must be whole swizzle atoms");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

template <int DT, int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmSA, const __grid_constant__ CUtensorMap tmSB,
                        const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ EpiMaps pm,
                        TcParams p) {
  using C = Cfg2<DT, BN, STAGES>;
  using T = typename C::T;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + C::BAR_OFF);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();             // 0 = leader
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_items = C::HALVES ? p.num_items : p.tiles_m * p.tiles_n;   // tiles of 256 x BN (or halves)
  AbortCtl ctl{p.dev_err, &bars->abort_flag};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);                     // the leader arms it for both CTAs
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 2 * 4);            // one arrival per epilogue warp, both CTAs
    }
    if constexpr (C::SCALED) {
      for (int st = 0; st < STAGES; ++st) mbar_init(&bars->sf_ready[st], 1);   // leader's copier
      for (int sl = 0; sl < C::SF_SLOTS; ++sl) mbar_init(&bars->sf_free[sl], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if constexpr (C::SCALED) {
    // 512 bytes of UE8M0 127 (scale 1) for an operand without a scale plane
    if (warp == 2)
      *reinterpret_cast<uint4*>(smem + C::SF_CONST_OFF + lane * 16) =
          make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  bool aborted_any = false;

  if (warp == 0 && lane == 0) {
    // ------------------------ TMA producer (both CTAs) ------------------------
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    // bytes each CTA lands per stage (the leader expects both CTAs' on its barrier)
    const uint32_t tx = C::STAGE_TX + (C::SCALED ? (p.sfa ? C::SF_A_BYTES : 0) + (p.sfb ? C::SF_B_BYTES : 0) : 0);
    if constexpr (C::SCALED) {
      tma_prefetch_desc(&tmSA);
      tma_prefetch_desc(&tmSB);
    }
    if constexpr (C::HALVES && !T::b_mn) tma_prefetch_desc(&tmBh);
    for (int item = pair; item < num_items && ok; item += npairs) {
      int tm, tn, half;
      item_coords(item, p, tm, tn, half);
      if constexpr (!C::HALVES) half = -1;
      // W columns this CTA loads: BH of the tile, or BH/2 of one half of it
      const int wcol = tn * BN + (half < 0 ? (int)rank * C::BH : half * (BN / 2) + (int)rank * (C::BH / 2));
      const uint32_t stx = half < 0 ? tx : (uint32_t)C::STAGE_TX_H;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&bars->empty[stage], phase ^ 1u, ctl, 0x100 + stage)) { ok = false; break; }
        const uint32_t lfull = mapa_shared(&bars->full[stage], 0);
        unsigned char* a_dst = smem + stage * C::STAGE_BYTES;
        unsigned char* b_dst = a_dst + C::A_BYTES;
        // Only the leader arrives, expecting both CTAs' bytes; the peer's loads
        // just complete their transactions on the leader's barrier (a remote
        // arrive per stage would put a cross-SM round trip in the peer's loop).
        if (rank == 0) mbar_arrive_expect_tx(&bars->full[stage], 2 * stx);
        // x counts elements of the map: 16-bit elements, else bytes
        tma_load_2d_pair(a_dst, &tmA, lfull,
                         kb * (T::a_bits == 16 ? C::K_PER_STAGE : kRowBytes),
                         tm * 256 + (int)rank * kBM);
        if constexpr (C::SCALED) {
          // packed scale blocks: rows of 512 bytes, [128-row tile][stage][cell]
          unsigned char* sf = smem + C::SF_OFF + stage * C::SF_STAGE_BYTES;
          if (p.sfa)
            tma_load_2d_pair(sf, &tmSA, lfull, 0, ((2 * tm + (int)rank) * p.num_kb + kb) * C::SF_CELLS);
          if (p.sfb) {
#pragma unroll
            for (int c = 0; c < C::SF_B_CHUNKS; ++c)
              tma_load_2d_pair(sf + C::SF_A_BYTES + c * C::SF_A_BYTES, &tmSB, lfull, 0,
                               ((tn * C::SF_B_CHUNKS + c) * p.num_kb + kb) * C::SF_CELLS);
          }
        }
        if constexpr (T::b_mn) {
          const int boxes = half < 0 ? C::B_BOXES : C::B_BOXES / 2;
#pragma unroll
          for (int j = 0; j < C::B_BOXES; ++j)
            if (j < boxes)
              tma_load_2d_pair(b_dst + j * C::B_BOX_BYTES, &tmB, lfull, wcol + j * C::B_BOX_MN, kb * C::K_PER_STAGE);
        } else {
          if (half < 0)
            tma_load_2d_pair(b_dst, &tmB, lfull, kb * (C::B_UNPACK ? C::K_PER_STAGE : kRowBytes), wcol);
          else   // a half tile: the half-height box of the same rows
            tma_load_2d_pair(b_dst, &tmBh, lfull, kb * kRowBytes, wcol);
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
    aborted_any = !ok;
  } else if (C::SCALED && warp == 3 && lane == 0 && rank == 0) {
    // --------------- scale-cell copier (block-scaled kinds, leader only) ---------
    // A stage's scale blocks go to both CTAs' TMEM with tcgen05.cp.cta_group::2
    // from this thread, committed to the leader's sf_ready barrier, on which the
    // MMA issuer waits in place of `full`.  Copying them in the MMA thread's own
    // loop measured 7-14 % slower: that single thread paces the scaled tiles.
    // (an operand without a scale plane has unit cells, which the MMA issuer
    // copies into every slot once; with no plane at all this thread has no work)
    // (with fewer TMEM slots than stages, a slot is rewritten once the MMAs of
    // the stage that last used it have completed: sf_free)
    uint32_t stage = 0, phase = 0, slot = 0, sphase = 0;
    bool ok = true;
    const bool work = p.sfa || p.sfb;
    const uint32_t smem_base = smem_u32(smem);
    for (int item = pair; work && item < num_items && ok; item += npairs) {
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&bars->full[stage], phase, ctl, 0x500 + stage)) { ok = false; break; }
        if constexpr (C::SF_SLOTS < STAGES)
          if (!mbar_wait(&bars->sf_free[slot], sphase ^ 1u, ctl, 0x600 + slot)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sf_smem = smem_base + C::SF_OFF + stage * C::SF_STAGE_BYTES;
        const uint32_t sf_tmem = tmem_base + (uint32_t)(C::SF_COL0 + slot * C::SF_COLS_STAGE);
#pragma unroll
        for (int g = 0; g < C::SF_CELLS; ++g) {
          const uint32_t sfa_t = sf_tmem + g * (C::SF_COLS_A + C::SF_COLS_B);
          if (p.sfa) tc_cp_pair_32x128b_warpx4(sfa_t, sdesc_plain(sf_smem + g * kSfChunk, 0, 128));
          if (p.sfb) {
#pragma unroll
            for (int c = 0; c < C::SF_B_CHUNKS; ++c)
              tc_cp_pair_32x128b_warpx4(sfa_t + C::SF_COLS_A + 4 * c,
                                        sdesc_plain(sf_smem + C::SF_A_BYTES + (c * C::SF_CELLS + g) * kSfChunk, 0,
                                                    128));
          }
        }
        tc_commit_pair(&bars->sf_ready[stage], 0x1);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        if (++slot == (uint32_t)C::SF_SLOTS) { slot = 0; sphase ^= 1u; }
      }
    }
    aborted_any = !ok;
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------ MMA issuer (leader only) ------------------------
    uint32_t stage = 0, phase = 0;
    int local = 0;
    bool ok = true;
    const uint32_t smem_base = smem_u32(smem);
    if constexpr (C::SCALED) {
      // unit scale cells (the block of 127s) for an operand without a scale
      // plane go into every ring slot of both CTAs once; this thread's MMAs
      // follow them in issue order
      const uint32_t sf_const = smem_base + C::SF_CONST_OFF;
      for (int st = 0; st < C::SF_SLOTS; ++st) {
        const uint32_t sf_tmem = tmem_base + (uint32_t)(C::SF_COL0 + st * C::SF_COLS_STAGE);
#pragma unroll
        for (int g = 0; g < C::SF_CELLS; ++g) {
          const uint32_t sfa_t = sf_tmem + g * (C::SF_COLS_A + C::SF_COLS_B);
          if (!p.sfa) tc_cp_pair_32x128b_warpx4(sfa_t, sdesc_plain(sf_const, 0, 128));
          if (!p.sfb) {
#pragma unroll
            for (int c = 0; c < C::SF_B_CHUNKS; ++c)
              tc_cp_pair_32x128b_warpx4(sfa_t + C::SF_COLS_A + 4 * c, sdesc_plain(sf_const, 0, 128));
          }
        }
      }
    }
    const bool via_copier = C::SCALED && (p.sfa || p.sfb);
    uint32_t slot = 0;   // TMEM scale slot of the stage
    for (int item = pair; item < num_items && ok; item += npairs, ++local) {
      const int buf = C::ACC_BUFS == 2 ? (local & 1) : 0;
      const uint32_t acc_par = C::ACC_BUFS == 2 ? (uint32_t)(local >> 1) & 1u : (uint32_t)local & 1u;
      if (!mbar_wait(&bars->acc_empty[buf], acc_par ^ 1u, ctl, 0x200 + buf)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
      const uint32_t idesc = (C::HALVES && item >= p.split_from) ? C::IDESC_H : C::IDESC;   // N = BN/2 for a half
      for (int kb = 0; kb < p.num_kb; ++kb) {
        // block-scaled kinds: the copier has also put the stage's scale cells in TMEM
        uint64_t* ready = via_copier ? &bars->sf_ready[stage] : &bars->full[stage];
        if (!mbar_wait(ready, phase, ctl, 0x300 + stage)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_base + stage * C::STAGE_BYTES;
        const uint32_t b_addr = a_addr + C::A_BYTES;
        if constexpr (C::SCALED) {
          const uint32_t sf_tmem = tmem_base + (uint32_t)(C::SF_COL0 + slot * C::SF_COLS_STAGE);
#pragma unroll
          for (int kk = 0; kk < C::MMAS_PER_STAGE; ++kk) {
            constexpr int per_cell = 4 / T::nsf;
            const int g = kk / per_cell;
            const uint32_t sfid = (uint32_t)((kk % per_cell) * T::nsf);
            const uint32_t sfa_t = sf_tmem + g * (C::SF_COLS_A + C::SF_COLS_B);
            const uint64_t adesc = sdesc_sw128(a_addr + kk * C::MMA_K_BYTES, 16, 1024);
            const uint64_t bdesc = sdesc_sw128(b_addr + kk * C::B_ADV, C::B_LBO, 1024);
            tc_mma_pair_bs<T::kind>(d_tmem, adesc, bdesc, C::IDESC | (sfid << 4) | (sfid << 29),
                                    (kb | kk) != 0 ? 1u : 0u, sfa_t, sfa_t + C::SF_COLS_A);
          }
        } else {
#pragma unroll
          for (int kk = 0; kk < C::MMAS_PER_STAGE; ++kk) {
            const uint64_t adesc = sdesc_sw128(a_addr + kk * C::MMA_K_BYTES, 16, 1024);
            const uint64_t bdesc = sdesc_sw128(b_addr + kk * C::B_ADV, C::B_LBO, 1024);
            tc_mma_pair<T::kind>(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
        }
        tc_commit_pair(&bars->empty[stage], 0x3);
        if constexpr (C::SCALED && C::SF_SLOTS < STAGES) {
          if (via_copier) tc_commit_pair(&bars->sf_free[slot], 0x1);   // this slot's MMAs, then its reuse
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        if constexpr (C::SCALED) {
          if (++slot == (uint32_t)C::SF_SLOTS) slot = 0;
        }
      }
      if (!ok) break;
      tc_commit_pair(&bars->acc_full[buf], 0x3);
    }
    aborted_any = !ok;
  } else if (warp >= 4) {
    // ------------------------ epilogue (both CTAs) ----------------------------
    const int q = warp - 4;
    int local = 0;
    int nst = 0;   // chunks this warp has stored through the TMA
    for (int item = pair; item < num_items; item += npairs, ++local) {
      int tm, tn, half;
      item_coords(item, p, tm, tn, half);
      if constexpr (!C::HALVES) half = -1;
      const int buf = C::ACC_BUFS == 2 ? (local & 1) : 0;
      const uint32_t acc_par = C::ACC_BUFS == 2 ? (uint32_t)(local >> 1) & 1u : (uint32_t)local & 1u;
      const bool got = mbar_wait(&bars->acc_full[buf], acc_par, ctl, 0x400 + buf);
      if (!__all_sync(0xffffffffu, got)) { aborted_any = true; break; }
      __syncwarp();
      tc_fence_after();
      const int row = tm * 256 + (int)rank * kBM + q * 32 + lane;
      const int col0 = tn * BN + (half > 0 ? BN / 2 : 0);
      const bool row_ok = row < p.N;
      uint32_t* yrow = reinterpret_cast<uint32_t*>(p.Y) + (size_t)row * p.M;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      auto release = [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(&bars->acc_empty[buf], 0));
      };
      unsigned char* epi = C::EPI_TMA ? smem + C::EPI_OFF + q * C::EPI_BUFS * 4096 : nullptr;
      // a half tile drains BN/64 chunks (only tiles that split have a half-tile path)
      bool halved = false;
      if constexpr (C::HALVES) {
        if (half >= 0) {
          halved = true;
          if (C::EPI_TMA && p.y_tma)
            drain_quadrant_tma<BN / 64, (C::EPI_BUFS > 0 ? C::EPI_BUFS : 1)>(taddr, col0, row - lane, p, release,
                                                                             epi, &pm, nst);
          else
            drain_quadrant<BN / 64>(taddr, yrow, col0, p.M, row_ok, p.col_exp, p, row - lane, release, epi, &pm);
        }
      }
      if (halved) continue;
      if constexpr (C::EPI_TMA) {
        if (p.y_tma) {
          drain_quadrant_tma<BN / 32, C::EPI_BUFS>(taddr, col0, row - lane, p, release, epi, &pm, nst);
          continue;
        }
      }
      drain_quadrant<BN / 32>(taddr, yrow, col0, p.M, row_ok, p.col_exp, p, row - lane, release, epi, &pm);
    }
    // TMA stores still in flight complete before the CTA ends
    if (C::EPI_TMA && (p.npeers || p.y_tma) && lane == 0) bulk_wait_all();
    __syncwarp();
  }

  if (aborted_any || aborted(ctl)) {
    // let TMA copies still in flight (ours or the peer's) land before exiting
    const unsigned long long t0 = global_ns();
    while (global_ns() - t0 < 100000ull) {}
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ----------------------------------------------------------------------------
// A16 widen kernel: fp16 activations x int8 / E4M3 / MXFP4 weights.
//
// The reference's W8A16 and MXFP4 (A16) kernels feed a half x {int8, E4M3,
// E2M1 + UE8M0} matmul2d (fp8_mlp.metal:127-164, :199-276).  Here the weights
// stay low-bit in HBM and shared memory: TMA brings the raw W tile of each
// stage into a staging buffer, four converter warps widen it exactly to f16
// straight into the 128-byte-swizzled UMMA layout, and the MMA runs
// kind::f16 (F16 x F16 -> F32).  Warps: 0 TMA, 1 MMA, 4-7 epilogue, 8-11
// converters (384 threads).
//
// Exactness: int8 -> f16 (|v| <= 128) and E4M3 -> f16 (cvt.rn.f16x2.e4m3x2)
// are exact.  E2M1 * 2^(s-127) is an f16 value only for s in [104, 140]; a
// pre-pass finds for every weight row m an exponent offset c_m that moves
// the row's scales into that window (0 for ordinary planes), the converters
// widen E2M1 * 2^(s-127-c_m) and the epilogue multiplies column m by 2^c_m.
// ----------------------------------------------------------------------------
constexpr int kWThreads = 384;

template <int DT>
struct WTraits {
  static constexpr bool mx = (DT == kMXFP4);
  static constexpr bool b_mn = !mx;   // int8 / E4M3 W is [K,M]
};

template <int DT, int BN, int STAGES>
struct WCfg {
  using WT = WTraits<DT>;
  static constexpr int A_BYTES = kBM * kRowBytes;            // 128 rows x 64 halfs
  static constexpr int B_BYTES = BN * kRowBytes;             // widened f16 tile
  static constexpr int K_PER_STAGE = 64;
  static constexpr int RAW_BYTES = WT::mx ? BN * 32 : K_PER_STAGE * BN;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + RAW_BYTES;
  static constexpr int STAGE_TX = A_BYTES + RAW_BYTES;
  static constexpr int MMAS_PER_STAGE = 4;                   // K = 16 each
  static constexpr uint32_t B_LBO = WT::b_mn ? 64u * kRowBytes : 16u;
  static constexpr uint32_t B_ADV = WT::b_mn ? 16u * kRowBytes : 32u;
  static constexpr uint32_t TMEM_COLS = pow2_cols(2 * BN);
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + kBarBytes + 1024;
  static constexpr uint32_t IDESC = (1u << 4) | (0u << 7) | (0u << 10) | ((WT::b_mn ? 1u : 0u) << 16) |
                                    ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
  static_assert(STAGE_BYTES % 1024 == 0, "swizzle atoms need 1 KB alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

struct WBars {
  uint64_t full[8];
  uint64_t conv[8];
  uint64_t empty[8];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct WParams {
  void* Y;
  const uint8_t* wscale;     // mxfp4: [M, K/32]
  const int8_t* col_exp;     // mxfp4: per-row exponent offsets c_m (from the pre-pass)
  int N, K, M;
  int tiles_m, tiles_n, num_kb;
  int* dev_err;
};

// Per weight row: the exponent offset c_m that brings the row's UE8M0 scales
// into the window where E2M1 * 2^(s-127-c_m) is an exact f16 (s in [104,140]).
__global__ void __launch_bounds__(256) mx_row_exp_kernel(const uint8_t* __restrict__ wscale, int M,
                                                         int kbpr, int8_t* __restrict__ out) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  int mn = 255, mx = 0;
  for (int i = lane; i < kbpr; i += 32) {
    const int s = wscale[(size_t)row * kbpr + i];
    mn = min(mn, s);
    mx = max(mx, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  int c = 0;
  if (mx > 140) c = mx - 140;
  else if (mn < 104) c = max(mn - 104, mx - 140);
  if (lane == 0) out[row] = (int8_t)c;
}

template <int DT, int BN, int STAGES>
__global__ void __launch_bounds__(kWThreads, 1)
    tc_widen_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmR,
                    WParams p) {
  using C = WCfg<DT, BN, STAGES>;
  using WT = typename C::WT;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  WBars* bars = reinterpret_cast<WBars*>(smem + C::BAR_OFF);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;
  AbortCtl ctl{p.dev_err, &bars->abort_flag};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->conv[s], 4);      // one arrival per converter warp
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 4 * 32);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmR);
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
        unsigned char* base = smem + stage * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&bars->full[stage], C::STAGE_TX);
        tma_load_2d(base, &tmA, &bars->full[stage], kb * C::K_PER_STAGE, tm * kBM);
        unsigned char* raw = base + C::A_BYTES + C::B_BYTES;
        if constexpr (WT::mx) tma_load_2d(raw, &tmR, &bars->full[stage], kb * 32, tn * BN);
        else tma_load_2d(raw, &tmR, &bars->full[stage], tn * BN, kb * C::K_PER_STAGE);
        filled[stage] = true;
        filled_parity[stage] = phase;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
    if (!ok) {
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
      const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&bars->full[stage], phase, ctl, 0x300 + stage) ||
            !mbar_wait(&bars->conv[stage], phase, ctl, 0x600 + stage)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_base + stage * C::STAGE_BYTES;
        const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < C::MMAS_PER_STAGE; ++kk) {
          const uint64_t adesc = sdesc_sw128(a_addr + kk * 32, 16, 1024);
          const uint64_t bdesc = sdesc_sw128(b_addr + kk * C::B_ADV, C::B_LBO, 1024);
          tc_mma<kKindF16>(d_tmem, adesc, bdesc, C::IDESC, (kb | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&bars->empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      tc_commit(&bars->acc_full[buf]);
    }
  } else if (warp >= 8) {
    // ------------------------------ converters --------------------------------
    const int ct = threadIdx.x - 256;   // 0..127
    const int kbpr = p.K / 32;
    uint32_t stage = 0, phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, tm, tn);
      (void)tm;
      bool ok = true;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const bool got = mbar_wait(&bars->full[stage], phase, ctl, 0x700 + stage);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        unsigned char* bconv = smem + stage * C::STAGE_BYTES + C::A_BYTES;
        const unsigned char* raw = bconv + C::B_BYTES;
        if constexpr (WT::mx) {
          // row n: 32 raw bytes (64 E2M1) -> 8 swizzled 16-byte chunks of f16
#pragma unroll
          for (int r = 0; r < BN / 128; ++r) {
            const int n = ct + 128 * r;
            const int m = tn * BN + n;
            uint32_t mul0 = 0, mul1 = 0;
            if (m < p.M) {
              const int c_m = p.col_exp[m];
              const uint8_t* sp = p.wscale + (size_t)m * kbpr + kb * 2;
              const int s0 = __ldg(sp);
              const int s1 = (kb * 2 + 1 < kbpr) ? __ldg(sp + 1) : 127;
              mul0 = f16x2_pow2(s0 - 127 - c_m);
              mul1 = f16x2_pow2(s1 - 127 - c_m);
            }
            const uint4 w0 = *reinterpret_cast<const uint4*>(raw + n * 32);
            const uint4 w1 = *reinterpret_cast<const uint4*>(raw + n * 32 + 16);
            const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            unsigned char* row = bconv + n * kRowBytes;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 h = widen_e2m1x8(words[c], c < 4 ? mul0 : mul1);
              *reinterpret_cast<uint4*>(row + ((c ^ (n & 7)) << 4)) = h;
            }
          }
        } else {
          // [64 K rows][BN] bytes -> BN/64 boxes of [64 K rows][128 B] f16
          constexpr int CHUNKS = C::K_PER_STAGE * BN / 8;
          constexpr int JB = BN / 64;
#pragma unroll 4
          for (int i = ct; i < CHUNKS; i += 128) {
            const int c = i & 7, rest = i >> 3;
            const int j = rest % JB, k = rest / JB;
            const uint2 v = *reinterpret_cast<const uint2*>(raw + k * BN + j * 64 + c * 8);
            const uint4 h = (DT == kINT8) ? widen_i8x8(v) : widen_e4m3x8(v);
            *reinterpret_cast<uint4*>(bconv + j * (64 * kRowBytes) + k * kRowBytes + ((c ^ (k & 7)) << 4)) = h;
          }
        }
        fence_proxy_async_smem();   // generic-proxy writes -> visible to tcgen05.mma
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->conv[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------ epilogue ----------------------------------
    const int q = warp - 4;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, tm, tn);
      const int buf = local & 1;
      const uint32_t acc_par = (uint32_t)(local >> 1) & 1u;
      const bool got = mbar_wait(&bars->acc_full[buf], acc_par, ctl, 0x400 + buf);
      if (!__all_sync(0xffffffffu, got)) break;
      __syncwarp();
      tc_fence_after();
      const int row = tm * kBM + q * 32 + lane;
      const int col0 = tn * BN;
      const bool row_ok = row < p.N;
      float* yrow = reinterpret_cast<float*>(p.Y) + (size_t)row * p.M;
      const bool vec_ok = (p.M % 4) == 0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + c * 32), r);
        tmem_ld_wait();
        const int cb = col0 + c * 32;
        float v[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) v[t] = __uint_as_float(r[t]);
        if constexpr (WT::mx) {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int m = cb + t;
            const int e = (m < p.M) ? p.col_exp[m] : 0;
            if (e) v[t] *= __int_as_float((e + 127) << 23);   // exact power of two
          }
        }
        if (row_ok) {
          if (vec_ok && cb + 32 <= p.M) {
            float4* dst = reinterpret_cast<float4*>(yrow + cb);
#pragma unroll
            for (int t = 0; t < 8; ++t) dst[t] = make_float4(v[4 * t], v[4 * t + 1], v[4 * t + 2], v[4 * t + 3]);
          } else {
#pragma unroll
            for (int t = 0; t < 32; ++t)
              if (cb + t < p.M) yrow[cb + t] = v[t];
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
// A16 kinds on CTA pairs: the [K,M] int8 / E4M3 weights are widened once per
// call to f16 in the workspace (exact), and the fp16 pair kernel runs on them.
// At the fat shape the widening (one read of W, one write of twice its bytes)
// costs about a tenth of the GEMM, whereas the converter warps of the widen
// kernel redo it for every 128 rows of X.
// ----------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) widen_w_f16_kernel(const uint8_t* __restrict__ W, uint4* __restrict__ out,
                                                          long n16) {
  // four 16-byte loads in flight per thread before any is converted
  constexpr int U = 4;
  const long stride = (long)gridDim.x * 256L;
  for (long i0 = blockIdx.x * 256L + threadIdx.x; i0 < n16; i0 += U * stride) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long i = i0 + u * stride;
      v[u] = i < n16 ? __ldcs(reinterpret_cast<const uint4*>(W) + i) : make_uint4(0, 0, 0, 0);   // read once
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long i = i0 + u * stride;
      if (i >= n16) break;
      const uint2 lo = make_uint2(v[u].x, v[u].y), hi = make_uint2(v[u].z, v[u].w);
      out[2 * i] = DT == kINT8 ? widen_i8x8(lo) : widen_e4m3x8(lo);
      out[2 * i + 1] = DT == kINT8 ? widen_i8x8(hi) : widen_e4m3x8(hi);
    }
  }
}

// mxfp4 weights [M,K] widened once to f16 in the [K,M] layout of the fp16
// weights (the pair kernel then reads them MN-major, its fastest form).  A block
// covers 128 rows x 64 K: each thread widens one 32-element block of one row
// (row offsets c_m from mx_row_exp_kernel) into a shared [64 K][128] tile, which
// goes out as 64 coalesced 256-byte rows of W16.
constexpr int kWtM = 128, kWtK = 64;

__global__ void __launch_bounds__(256) widen_mx_t_kernel(const uint8_t* __restrict__ W,
                                                         const uint8_t* __restrict__ wscale,
                                                         const int8_t* __restrict__ col_exp, int M, int K,
                                                         __half* __restrict__ out) {
  __shared__ __align__(16) __half tile[kWtK][kWtM];
  const int t = threadIdx.x, r = t & 127, q = t >> 7;   // row of the tile, which 32 K
  const int m0 = blockIdx.x * kWtM, k0 = blockIdx.y * kWtK;
  const int m = m0 + r, kb = k0 / 32 + q, kbpr = K / 32;
  uint32_t h[16];
  if (m < M && kb < kbpr) {
    const uint4 w = __ldcs(reinterpret_cast<const uint4*>(W + (size_t)m * (K / 2)) + kb);
    const uint32_t mul = f16x2_pow2((int)__ldg(wscale + (size_t)m * kbpr + kb) - 127 - (int)col_exp[m]);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = widen_e2m1x8(words[i], mul);
      h[4 * i] = v.x;
      h[4 * i + 1] = v.y;
      h[4 * i + 2] = v.z;
      h[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) h[i] = 0;
  }
  // element k = 32 q + 2 i (+1) of row r; a warp writes 32 consecutive rows per K
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    tile[32 * q + 2 * i][r] = __ushort_as_half((unsigned short)(h[i] & 0xFFFFu));
    tile[32 * q + 2 * i + 1][r] = __ushort_as_half((unsigned short)(h[i] >> 16));
  }
  __syncthreads();
  // 64 K rows x 16 chunks of 8 f16 (M % 8 == 0)
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int i = t + 256 * it, c = i & 15, kr = i >> 4;
    const int k = k0 + kr, mc = m0 + 8 * c;
    if (k < K && mc < M)
      *reinterpret_cast<uint4*>(out + (size_t)k * M + mc) = *reinterpret_cast<const uint4*>(&tile[kr][8 * c]);
  }
}

}  // namespace

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

// 2-D row-major map: `inner` elements per row (contiguous), `outer` rows,
// `row_bytes` between rows.
bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType ty, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, ty, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Same, without swizzle (raw weight tiles read by the converter warps).
bool make_map_plain(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Packed scale blocks (sf_pack_kernel output) as a 2-D map: `rows` rows of
// 128 x 32-bit (one 512-byte block each), boxes of `cells` rows, no swizzle.
bool make_map_sf(CUtensorMap* m, const void* base, uint64_t rows, uint32_t cells) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {128, rows};
  cuuint64_t strides[1] = {(cuuint64_t)kSfChunk};
  cuuint32_t box[2] = {128, cells};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

bool aligned(const void* p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// One-time set-up of a kernel per device (the dynamic shared-memory opt-in and,
// for the pair kernel, its co-resident cluster count).  The lock keeps host
// threads that launch on the same device at the same time from racing on it.
struct DevOnce {
  std::mutex mu;
  unsigned mask = 0;      // bit d: device d is set up
  int value[32] = {0};    // per-device result (max co-resident CTA pairs)
};

template <int DT, int BN, int STAGES>
cudaError_t launch_cfg(const RunArgs& a, const void* W, const uint8_t* sfa = nullptr,
                       const uint8_t* sfb = nullptr) {
  using C = Cfg<DT, BN, STAGES>;
  using T = typename C::T;
  CUtensorMap tmA, tmB;
  const CUtensorMapDataType ty8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  bool ok;
  if constexpr (T::a_bits == 16) {
    ok = make_map(&tmA, a.X, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)a.K, (uint64_t)a.N,
                  (uint64_t)a.K * 2, C::K_PER_STAGE, kBM);
  } else {
    const uint64_t row_bytes = (uint64_t)a.K * T::a_bits / 8;
    ok = make_map(&tmA, a.X, ty8, row_bytes, (uint64_t)a.N, row_bytes, kRowBytes, kBM);
  }
  if (!ok) return cudaErrorInvalidValue;
  if constexpr (T::b_mn) {
    const int es = T::b_bits / 8;
    ok = make_map(&tmB, W, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : ty8, (uint64_t)a.M, (uint64_t)a.K,
                  (uint64_t)a.M * es, C::B_BOX_MN, C::K_PER_STAGE);
  } else if constexpr (T::b_unpack4) {
    // packed E2M1 [M,K] -> 8-bit containers in shared memory (16 values + 8 bytes gap)
    ok = make_map(&tmB, W, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, (uint64_t)a.K, (uint64_t)a.M,
                  (uint64_t)a.K / 2, 128, BN);
  } else {
    const uint64_t row_bytes = (uint64_t)a.K * T::b_bits / 8;
    ok = make_map(&tmB, W, ty8, row_bytes, (uint64_t)a.M, row_bytes, kRowBytes, BN);
  }
  if (!ok) return cudaErrorInvalidValue;

  TcParams p;
  p.Y = a.Y;
  p.sfa = sfa;
  p.sfb = sfb;
  p.col_exp = nullptr;
  p.N = a.N;
  p.K = a.K;
  p.M = a.M;
  p.tiles_m = (a.N + kBM - 1) / kBM;
  p.tiles_n = (a.M + BN - 1) / BN;
  p.num_kb = (a.K + C::K_PER_STAGE - 1) / C::K_PER_STAGE;
  p.dev_err = a.dev_err;
  set_peers(p, a);
  const int tiles = p.tiles_m * p.tiles_n;
  p.split_from = p.num_items = tiles;   // whole tiles only
  // the TMA-store epilogue wherever Y's rows are whole 16-byte units
  EpiMaps em;
  std::memset(&em, 0, sizeof(em));
  p.y_tma = (a.M % 4 == 0 && aligned(a.Y, 16)) ? 1 : 0;
  if (p.y_tma) {
    if (!make_map(&em.y, a.Y, CU_TENSOR_MAP_DATA_TYPE_UINT32, (uint64_t)a.M, (uint64_t)a.N, (uint64_t)a.M * 4, 32, 32))
      return cudaErrorInvalidValue;
    for (int i = 0; i < a.npeers; ++i)
      if (!make_map(&em.m[i], a.ypeers[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, (uint64_t)a.M, (uint64_t)a.N,
                    (uint64_t)a.M * 4, 32, 32))
        return cudaErrorInvalidValue;
  }
  const int grid = tiles < a.num_sms ? tiles : a.num_sms;
  auto k = tc_gemm_kernel<DT, BN, STAGES>;
  static DevOnce once;   // per device: dynamic shared memory opt-in done
  const int dev = current_device();
  {
    std::lock_guard<std::mutex> lk(once.mu);
    if (!(once.mask & (1u << (dev & 31)))) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_EPI);
      if (e != cudaSuccess) return e;
      once.mask |= 1u << (dev & 31);
    }
  }
  k<<<grid, kThreads, p.y_tma ? C::SMEM_EPI : C::SMEM_BYTES, a.stream>>>(tmA, tmB, em, p);
  return cudaGetLastError();
}

template <int DT, int BN, int STAGES>
cudaError_t launch_pair(const RunArgs& a, const void* W, const uint8_t* sfa = nullptr, const uint8_t* sfb = nullptr,
                        int sf_rows_a = 0, int sf_rows_b = 0, const int8_t* col_exp = nullptr) {
  using C = Cfg2<DT, BN, STAGES>;
  using T = typename C::T;
  CUtensorMap tmA, tmB, tmSA, tmSB;
  const CUtensorMapDataType ty8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  bool ok;
  if constexpr (T::a_bits == 16) {
    ok = make_map(&tmA, a.X, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K * 2,
                  C::K_PER_STAGE, kBM);
  } else {
    const uint64_t row_bytes = (uint64_t)a.K * T::a_bits / 8;
    ok = make_map(&tmA, a.X, ty8, row_bytes, (uint64_t)a.N, row_bytes, kRowBytes, kBM);
  }
  if (!ok) return cudaErrorInvalidValue;
  if constexpr (C::B_UNPACK) {
    ok = make_map(&tmB, W, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, (uint64_t)a.K, (uint64_t)a.M,
                  (uint64_t)a.K / 2, C::K_PER_STAGE, C::BH);
  } else if constexpr (T::b_mn) {
    const int es = T::b_bits / 8;
    ok = make_map(&tmB, W, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : ty8, (uint64_t)a.M, (uint64_t)a.K,
                  (uint64_t)a.M * es, C::B_BOX_MN, C::K_PER_STAGE);
  } else {
    const uint64_t row_bytes = (uint64_t)a.K * T::b_bits / 8;
    ok = make_map(&tmB, W, ty8, row_bytes, (uint64_t)a.M, row_bytes, kRowBytes, C::BH);
  }
  if (!ok) return cudaErrorInvalidValue;
  // half tiles (K-major W): the same rows in boxes of BH/2
  CUtensorMap tmBh = tmB;
  if constexpr (C::HALVES && !T::b_mn) {
    const uint64_t row_bytes = (uint64_t)a.K * T::b_bits / 8;
    if (!make_map(&tmBh, W, ty8, row_bytes, (uint64_t)a.M, row_bytes, kRowBytes, C::BH / 2))
      return cudaErrorInvalidValue;
  }
  // packed scale blocks as 2-D maps: rows of 128 x 32-bit (512 bytes), SF_CELLS rows per box
  tmSA = tmA;
  tmSB = tmA;
  if constexpr (C::SCALED) {
    if (sfa && !make_map_sf(&tmSA, sfa, (uint64_t)sf_rows_a, C::SF_CELLS)) return cudaErrorInvalidValue;
    if (sfb && !make_map_sf(&tmSB, sfb, (uint64_t)sf_rows_b, C::SF_CELLS)) return cudaErrorInvalidValue;
  }
  TcParams p;
  p.Y = a.Y;
  p.sfa = sfa;
  p.sfb = sfb;
  p.col_exp = col_exp;
  p.N = a.N;
  p.K = a.K;
  p.M = a.M;
  p.tiles_m = (a.N + 255) / 256;
  p.tiles_n = (a.M + BN - 1) / BN;
  p.num_kb = (a.K + C::K_PER_STAGE - 1) / C::K_PER_STAGE;
  p.dev_err = a.dev_err;
  set_peers(p, a);
  const int tiles = p.tiles_m * p.tiles_n;
  auto k = tc_gemm_pair_kernel<DT, BN, STAGES>;
  static DevOnce once;   // per device: shared-memory opt-in and co-resident CTA pairs (grid size)
  const int dev = current_device();
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int cap = 0;
  {
    std::lock_guard<std::mutex> lk(once.mu);
    if (!(once.mask & (1u << (dev & 31)))) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
      if (e != cudaSuccess) return e;
      int n = 0;
      cfg.gridDim = dim3(a.num_sms);
      if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess || n <= 0) n = a.num_sms / 2;
      once.value[dev & 31] = n;
      once.mask |= 1u << (dev & 31);
    }
    cap = once.value[dev & 31];
  }
  if (cap <= 0) cap = a.num_sms / 2;
  const int pairs = tiles < cap ? tiles : cap;
  // a last wave of at most half the pairs runs as twice as many half tiles
  const int rem = tiles % pairs;
  p.split_from = (C::HALVES && rem > 0 && 2 * rem <= pairs) ? tiles - rem : tiles;
  p.num_items = tiles + (tiles - p.split_from);
  // this GPU's and the peers' Y blocks as TMA store targets (rows of M 32-bit
  // words, a multiple of 16 bytes)
  EpiMaps pm;
  std::memset(&pm, 0, sizeof(pm));
  const bool use_epi = C::EPI_TMA && a.M % 4 == 0 && aligned(a.Y, 16);
  p.y_tma = use_epi ? 1 : 0;
  // the staging buffers are dynamic shared memory, requested only when used
  cfg.dynamicSmemBytes = use_epi ? C::SMEM_BYTES : C::SMEM_BASE;
  if (use_epi) {
    if (!make_map(&pm.y, a.Y, CU_TENSOR_MAP_DATA_TYPE_UINT32, (uint64_t)a.M, (uint64_t)a.N, (uint64_t)a.M * 4, 32, 32))
      return cudaErrorInvalidValue;
    for (int i = 0; i < a.npeers; ++i)
      if (!make_map(&pm.m[i], a.ypeers[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, (uint64_t)a.M, (uint64_t)a.N,
                    (uint64_t)a.M * 4, 32, 32))
        return cudaErrorInvalidValue;
  }
  cfg.gridDim = dim3(2 * pairs);
  return cudaLaunchKernelEx(&cfg, k, tmA, tmB, tmSA, tmSB, tmBh, pm, p);
}

template <int DT, int BN, int STAGES>
cudaError_t launch_widen(const RunArgs& a) {
  using C = WCfg<DT, BN, STAGES>;
  using WT = typename C::WT;
  CUtensorMap tmA, tmR;
  if (!make_map(&tmA, a.X, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K * 2,
                C::K_PER_STAGE, kBM))
    return cudaErrorInvalidValue;
  bool ok;
  if constexpr (WT::mx) {
    ok = make_map_plain(&tmR, a.W, (uint64_t)a.K / 2, (uint64_t)a.M, (uint64_t)a.K / 2, 32, BN);
  } else {
    ok = make_map_plain(&tmR, a.W, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.M, BN, C::K_PER_STAGE);
  }
  if (!ok) return cudaErrorInvalidValue;
  WParams p;
  p.Y = a.Y;
  p.wscale = a.wscale;
  p.col_exp = nullptr;
  p.N = a.N;
  p.K = a.K;
  p.M = a.M;
  p.tiles_m = (a.N + kBM - 1) / kBM;
  p.tiles_n = (a.M + BN - 1) / BN;
  p.num_kb = (a.K + C::K_PER_STAGE - 1) / C::K_PER_STAGE;
  p.dev_err = a.dev_err;
  if constexpr (WT::mx) {
    int8_t* ce = static_cast<int8_t*>(a.ws);
    mx_row_exp_kernel<<<(a.M + 7) / 8, 256, 0, a.stream>>>(a.wscale, a.M, a.K / 32, ce);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    p.col_exp = ce;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < a.num_sms ? tiles : a.num_sms;
  auto k = tc_widen_kernel<DT, BN, STAGES>;
  static DevOnce once;
  const int dev = current_device();
  {
    std::lock_guard<std::mutex> lk(once.mu);
    if (!(once.mask & (1u << (dev & 31)))) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
      if (e != cudaSuccess) return e;
      once.mask |= 1u << (dev & 31);
    }
  }
  k<<<grid, kWThreads, C::SMEM_BYTES, a.stream>>>(tmA, tmR, p);
  return cudaGetLastError();
}


}  // namespace

bool tc_supported(int dt, int bm, int bn, int N, int K, int M) {
  if (N <= 0 || K <= 0 || M <= 0) return false;
  if (bn == 192 || bn == 224) {   // CTA pairs, 256x192 / 256x224: the block-scaled kinds (two accumulators)
    if (bm != 256) return false;
    if (dt == kMX4X4) return K % 32 == 0;
    if (dt == kF4F4) return K % 32 == 0 && M % 2 == 0;
    if (dt == kMX8X4 || dt == kF8X4) return K % 128 == 0;
    return false;
  }
  if (bn != 128 && bn != 256) return false;
  if (bm == 256) {   // CTA-pair tiles: the unscaled kinds, 256-wide
    if (bn != 256) return false;
    if (dt == kFP16) return K % 8 == 0 && M % 8 == 0;
    if (dt == kINT8 || dt == kFP8) return K % 8 == 0 && M % 16 == 0;   // widened to f16 first
    if (dt == kMXFP4) return K % 32 == 0 && M % 8 == 0;                 // widened to f16 [K,M] first
    if (dt == kI8I8 || dt == kF8F8) return K % 16 == 0 && M % 16 == 0;
    if (dt == kF4F4) return K % 32 == 0 && M % 2 == 0;   // kind::f8f6f4 on unpacked E2M1
    if (dt == kMX4X4) return K % 32 == 0;                  // block-scaled kinds
    if (dt == kMX8X4 || dt == kF8X4) return K % 128 == 0;
    return false;
  }
  if (bm != 128) return false;
  switch (dt) {
    case kFP16: return K % 8 == 0 && M % 8 == 0;
    case kI8I8:
    case kF8F8: return K % 16 == 0 && M % 16 == 0;
    case kMX4X4: return K % 32 == 0;
    case kF4F4: return K % 32 == 0 && M % 2 == 0;
    case kMX8X4:
    case kF8X4: return K % 128 == 0;
    case kINT8:
    case kFP8: return K % 8 == 0 && M % 16 == 0;
    case kMXFP4: return K % 32 == 0;
    default: return false;
  }
}

namespace {

size_t round256(size_t x) { return (x + 255) / 256 * 256; }

// Workspace of the block-scaled kinds: [packed X scales][packed W scales]
// [f4f4: W transposed to [M,K]].
struct ScaledWs {
  size_t a_bytes = 0, b_bytes = 0, wt_bytes = 0;
  int stages = 0, a_tiles = 0, b_tiles = 0, nb = 0, cells = 0;
  int b_tile_rows = 0, b_chunks = 0;   // W rows per MMA tile (BN) and its 128-row chunks
  size_t total() const { return round256(a_bytes) + round256(b_bytes) + round256(wt_bytes); }
};

ScaledWs scaled_ws(int dt, int bn, int N, int K, int M) {
  ScaledWs w;
  const bool mxf4 = (dt == kMX4X4 || dt == kF4F4);
  const int kps = mxf4 ? 256 : 128;
  w.nb = kps / 32;
  w.cells = w.nb / 4;   // 32-bit cells of 4 k-blocks per stage
  w.stages = (K + kps - 1) / kps;
  w.a_tiles = (N + 127) / 128;
  w.b_tile_rows = bn;
  w.b_chunks = (bn + 127) / 128;
  w.b_tiles = (M + bn - 1) / bn * w.b_chunks;
  const bool xp = (dt == kMX4X4 || dt == kMX8X4), wp = (dt != kF4F4);
  if (xp) w.a_bytes = (size_t)w.a_tiles * w.stages * w.cells * kSfChunk;
  if (wp) w.b_bytes = (size_t)w.b_tiles * w.stages * w.cells * kSfChunk;
  if (dt == kF4F4) w.wt_bytes = (size_t)M * K / 2;
  return w;
}

bool is_scaled(int dt) { return dt == kMX4X4 || dt == kMX8X4 || dt == kF8X4 || dt == kF4F4; }

template <int DT, int BN, int STAGES>
cudaError_t launch_scaled(const RunArgs& a) {
  const ScaledWs w = scaled_ws(DT, BN, a.N, a.K, a.M);
  if (!a.ws || a.ws_bytes < w.total() || !aligned(a.ws, 256)) return cudaErrorInvalidValue;
  uint8_t* base = static_cast<uint8_t*>(a.ws);
  uint8_t* pa = w.a_bytes ? base : nullptr;
  uint8_t* pb = w.b_bytes ? base + round256(w.a_bytes) : nullptr;
  uint8_t* wt = base + round256(w.a_bytes) + round256(w.b_bytes);
  cudaError_t e;
  if (pa || pb) {
    SfPackJob ja{pa ? a.xscale : nullptr, pa, a.N, w.a_tiles, 128, 1};
    SfPackJob jb{pb ? a.wscale : nullptr, pb, a.M, w.b_tiles, w.b_tile_rows, w.b_chunks};
    const int tiles = w.a_tiles > w.b_tiles ? w.a_tiles : w.b_tiles;
    const int threads = tiles * w.stages * w.cells * 32;
    sf_pack_kernel<<<dim3((threads + 255) / 256, 2), 256, 0, a.stream>>>(ja, jb, a.K / 32, w.stages, w.nb, w.cells);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const void* W = a.W;
  if constexpr (DT == kF4F4) {
    dim3 grid((a.M + kTrM - 1) / kTrM, (a.K + kTrK - 1) / kTrK);
    transpose_fp4_kernel<<<grid, 256, 0, a.stream>>>(static_cast<const uint8_t*>(a.W), wt, a.K, a.M);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    W = wt;
  }
  return launch_cfg<DT, BN, STAGES>(a, W, pa, pb);
}

// Block-scaled kinds on CTA pairs (256x256 tiles): pack the scale planes into
// per-stage blocks (one 512-byte block per 128 rows and cell), then the pair
// kernel; each CTA brings its own rows' X scales and all 256 columns' W scales.
template <int DT, int BN>
cudaError_t launch_scaled_pair(const RunArgs& a) {
  // 5 stages leave room for two TMA-store staging buffers per epilogue warp.
  // mxfp4/a4 on 256x224 takes a sixth stage with one staging buffer: fat row
  // 68.8 against 70.8 us, square 56.5 against 58.4 us (same box, interleaved);
  // the same change measured even for f4f4 and a8 and slower for mxfp4/f8.
  constexpr int kStagesPair = (DT == kMX4X4 && BN == 224) ? 6 : 5;
  const ScaledWs w = scaled_ws(DT, BN, a.N, a.K, a.M);
  if (!a.ws || a.ws_bytes < w.total() || !aligned(a.ws, 256)) return cudaErrorInvalidValue;
  uint8_t* base = static_cast<uint8_t*>(a.ws);
  uint8_t* pa = w.a_bytes ? base : nullptr;
  uint8_t* pb = w.b_bytes ? base + round256(w.a_bytes) : nullptr;
  if (pa || pb) {
    SfPackJob ja{pa ? a.xscale : nullptr, pa, a.N, w.a_tiles, 128, 1};
    SfPackJob jb{pb ? a.wscale : nullptr, pb, a.M, w.b_tiles, w.b_tile_rows, w.b_chunks};
    const int tiles = w.a_tiles > w.b_tiles ? w.a_tiles : w.b_tiles;
    const int threads = tiles * w.stages * w.cells * 32;
    sf_pack_kernel<<<dim3((threads + 255) / 256, 2), 256, 0, a.stream>>>(ja, jb, a.K / 32, w.stages, w.nb, w.cells);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return launch_pair<DT, BN, kStagesPair>(a, a.W, pa, pb, w.a_tiles * w.stages * w.cells,
                                          w.b_tiles * w.stages * w.cells);
}

// f4f4 on CTA pairs: transpose W to [M,K] into the workspace (the 4-bit MMA
// operands are K-major), then kind::mxf4 (E2M1 x E2M1) with unit scales.
template <int BN>
cudaError_t launch_f4f4_pair(const RunArgs& a) {
  const ScaledWs w = scaled_ws(kF4F4, BN, a.N, a.K, a.M);
  if (!a.ws || a.ws_bytes < w.total() || !aligned(a.ws, 256)) return cudaErrorInvalidValue;
  uint8_t* wt = static_cast<uint8_t*>(a.ws) + round256(w.a_bytes) + round256(w.b_bytes);
  dim3 grid((a.M + kTrM - 1) / kTrM, (a.K + kTrK - 1) / kTrK);
  transpose_fp4_kernel<<<grid, 256, 0, a.stream>>>(static_cast<const uint8_t*>(a.W), wt, a.K, a.M);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // kind::mxf4 with unit scales (no scale planes: the kernel's block of UE8M0
  // 127s), on packed E2M1 straight from shared memory
  return launch_pair<kF4F4, BN, 5>(a, wt);
}

}  // namespace

size_t tc_workspace(int dt, int bm, int bn, int N, int K, int M) {
  if (is_scaled(dt)) return scaled_ws(dt, bn, N, K, M).total();
  if (bm == 256 && (dt == kINT8 || dt == kFP8)) return round256((size_t)K * M * 2);   // f16 copy of W
  if (bm == 256 && dt == kMXFP4) return round256((size_t)K * M * 2) + round256((size_t)M);   // + column offsets
  if (dt == kMXFP4) return (size_t)M + 256;          // per-row exponent offsets
  return 0;
}

int tc_launches(int dt, int bm) {
  if (bm == 256 && dt == kMXFP4) return 3;   // row offsets, widen, GEMM
  if (dt == kMXFP4 || dt == kF4F4 || dt == kMX4X4 || dt == kMX8X4 || dt == kF8X4) return 2;
  if (bm == 256 && (dt == kINT8 || dt == kFP8)) return 2;
  return 1;
}

namespace {

template <int DT>
cudaError_t launch_widened_pair(const RunArgs& a) {
  const size_t need = (size_t)a.K * a.M * 2;
  if (!a.ws || a.ws_bytes < need || !aligned(a.ws, 256)) return cudaErrorInvalidValue;
  const long n16 = (long)a.K * a.M / 16;   // M % 16 == 0
  long g = (n16 + 255) / 256;
  if (g > 8L * a.num_sms) g = 8L * a.num_sms;
  widen_w_f16_kernel<DT><<<(unsigned)g, 256, 0, a.stream>>>(static_cast<const uint8_t*>(a.W),
                                                           static_cast<uint4*>(a.ws), n16);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_pair<kFP16, 256, 6>(a, a.ws);
}

cudaError_t launch_widened_mx_pair(const RunArgs& a) {
  const size_t wbytes = round256((size_t)a.K * a.M * 2);
  if (!a.ws || a.ws_bytes < wbytes + round256((size_t)a.M) || !aligned(a.ws, 256)) return cudaErrorInvalidValue;
  __half* w16 = static_cast<__half*>(a.ws);
  int8_t* col_exp = static_cast<int8_t*>(a.ws) + wbytes;
  mx_row_exp_kernel<<<(a.M + 7) / 8, 256, 0, a.stream>>>(a.wscale, a.M, a.K / 32, col_exp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 grid((a.M + kWtM - 1) / kWtM, (a.K + kWtK - 1) / kWtK);
  widen_mx_t_kernel<<<grid, 256, 0, a.stream>>>(static_cast<const uint8_t*>(a.W), a.wscale, col_exp, a.M, a.K,
                                                w16);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_pair<kFP16, 256, 6>(a, w16, nullptr, nullptr, 0, 0, col_exp);
}

}  // namespace

bool tc_gather_supported(int dt, int bm) {
  return bm == 256 || !(dt == kINT8 || dt == kFP8 || dt == kMXFP4);
}

cudaError_t launch_tc(const RunArgs& a, int bm, int bn) {
  if (!tc_supported(a.dt, bm, bn, a.N, a.K, a.M)) return cudaErrorInvalidValue;
  if (a.npeers < 0 || a.npeers > kMaxPeers || (a.npeers && !tc_gather_supported(a.dt, bm)))
    return cudaErrorInvalidValue;
  for (int i = 0; i < a.npeers; ++i)
    if (!a.ypeers || !aligned(a.ypeers[i], 16)) return cudaErrorInvalidValue;
  if (!aligned(a.X, 16) || !aligned(a.W, 32) || !aligned(a.Y, 16)) return cudaErrorInvalidValue;
  if (bm == 256 && bn == 224) {   // block-scaled kinds, two accumulators (TMEM scale slots reused)
    switch (a.dt) {
      case kF4F4: return launch_f4f4_pair<224>(a);
      case kMX4X4: return launch_scaled_pair<kMX4X4, 224>(a);
      case kMX8X4: return launch_scaled_pair<kMX8X4, 224>(a);
      case kF8X4: return launch_scaled_pair<kF8X4, 224>(a);
      default: return cudaErrorInvalidValue;
    }
  }
  if (bm == 256 && bn == 192) {   // block-scaled kinds, two accumulators
    switch (a.dt) {
      case kF4F4: return launch_f4f4_pair<192>(a);
      case kMX4X4: return launch_scaled_pair<kMX4X4, 192>(a);
      case kMX8X4: return launch_scaled_pair<kMX8X4, 192>(a);
      case kF8X4: return launch_scaled_pair<kF8X4, 192>(a);
      default: return cudaErrorInvalidValue;
    }
  }
  if (bm == 256) {
    switch (a.dt) {
      case kFP16: return launch_pair<kFP16, 256, 6>(a, a.W);
      case kI8I8: return launch_pair<kI8I8, 256, 6>(a, a.W);
      case kF8F8: return launch_pair<kF8F8, 256, 6>(a, a.W);
      case kINT8: return launch_widened_pair<kINT8>(a);
      case kFP8: return launch_widened_pair<kFP8>(a);
      case kMXFP4: return launch_widened_mx_pair(a);
      case kF4F4: return launch_f4f4_pair<256>(a);
      case kMX4X4: return launch_scaled_pair<kMX4X4, 256>(a);
      case kMX8X4: return launch_scaled_pair<kMX8X4, 256>(a);
      case kF8X4: return launch_scaled_pair<kF8X4, 256>(a);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (a.dt) {
    case kFP16: return bn == 256 ? launch_cfg<kFP16, 256, 4>(a, a.W) : launch_cfg<kFP16, 128, 6>(a, a.W);
    case kI8I8: return bn == 256 ? launch_cfg<kI8I8, 256, 4>(a, a.W) : launch_cfg<kI8I8, 128, 6>(a, a.W);
    case kF8F8: return bn == 256 ? launch_cfg<kF8F8, 256, 4>(a, a.W) : launch_cfg<kF8F8, 128, 6>(a, a.W);
    case kINT8: return bn == 256 ? launch_widen<kINT8, 256, 3>(a) : launch_widen<kINT8, 128, 5>(a);
    case kFP8: return bn == 256 ? launch_widen<kFP8, 256, 3>(a) : launch_widen<kFP8, 128, 5>(a);
    case kMXFP4: {
      if (!a.ws || a.ws_bytes < tc_workspace(a.dt, bm, bn, a.N, a.K, a.M)) return cudaErrorInvalidValue;
      return bn == 256 ? launch_widen<kMXFP4, 256, 3>(a) : launch_widen<kMXFP4, 128, 5>(a);
    }
    case kMX4X4: return bn == 256 ? launch_scaled<kMX4X4, 256, 4>(a) : launch_scaled<kMX4X4, 128, 5>(a);
    case kMX8X4: return bn == 256 ? launch_scaled<kMX8X4, 256, 4>(a) : launch_scaled<kMX8X4, 128, 5>(a);
    case kF8X4: return bn == 256 ? launch_scaled<kF8X4, 256, 4>(a) : launch_scaled<kF8X4, 128, 5>(a);
    case kF4F4: return bn == 256 ? launch_scaled<kF4F4, 256, 4>(a) : launch_scaled<kF4F4, 128, 5>(a);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mlpg
