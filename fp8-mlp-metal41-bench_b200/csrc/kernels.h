// kernels.h -- internal launch interface between the C ABI (api.cu) and the
// kernel translation units.  Not part of the public boundary.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace mlpg {

struct RunArgs {
  int dt;
  const void* X;
  const void* W;
  void* Y;
  const uint8_t* xscale;
  const uint8_t* wscale;
  int N, K, M;
  void* ws;          // caller workspace (may be null when none is needed)
  size_t ws_bytes;
  cudaStream_t stream;
  int* dev_err;      // device error word (bounded-wait timeouts)
  int num_sms;
  // Fused all-gather: the tensor-core epilogue also stores every Y element at
  // the same offset from each of these peer base pointers (other GPUs' Y
  // buffers mapped into this context; see gemm_run_gather).
  void* const* ypeers = nullptr;
  int npeers = 0;
};

constexpr int kMaxPeers = 7;   // peers of one rank in an 8-GPU node

// ---- CUDA-core split-K GEMV (thin rows; also the any-shape fallback) --------
// Up to 8 K splits reduce inside a thread-block cluster (no workspace); more
// splits reduce through the workspace.
bool gemv_supported(int dt, int ksplit, int N, int K, int M);
int gemv_auto_ksplit(int dt, int N, int K, int M, int num_sms);
size_t gemv_workspace(int dt, int ksplit, int N, int K, int M);
cudaError_t launch_gemv(const RunArgs& a, int ksplit);

// ---- persistent TMA-streaming GEMV (thin rows, N <= 16) -------------------------
bool stream_supported(int dt, int N, int K, int M);
size_t stream_workspace(int dt, int N, int K, int M);
cudaError_t launch_stream(const RunArgs& a);

// ---- thin rows on the warp-level tensor-core MMA (gemv_mma.cu, tile "gemv.mma") --
// N <= 16 for fp16, int8, fp8, f8f8 ([K,M]) and the four MX kinds ([M,K]):
// persistent stream-K over slabs of the weights, mma.sync.m16n8k16 on weights
// widened to f16 in registers.  The workspace holds slab counters and partials.
bool mma_supported(int dt, int N, int K, int M);
size_t mma_workspace(int dt, int N, int K, int M);
cudaError_t launch_mma(const RunArgs& a);

// ---- thin rows on the tensor cores (N <= 16; weights as the MMA's A operand) ----
// Stream-K over (128-row weight tile, K stage) units, one CTA per SM; shared
// tiles are summed through the workspace (counters zero before first use).
bool thin_supported(int dt, int N, int K, int M);
size_t thin_workspace(int dt, int N, int K, int M);
cudaError_t launch_thin(const RunArgs& a);

// ---- tcgen05 tensor-core GEMM --------------------------------------------------
// bm: 128 (one CTA per tile) or 256 (a CTA pair, cta_group::2); bn: 128 or 256.
bool tc_supported(int dt, int bm, int bn, int N, int K, int M);
size_t tc_workspace(int dt, int bm, int bn, int N, int K, int M);
int tc_launches(int dt, int bm);
cudaError_t launch_tc(const RunArgs& a, int bm, int bn);
// Tiles whose epilogue can store to peer Y buffers as well (all but the
// 1-CTA converter-warp A16 kernel).
bool tc_gather_supported(int dt, int bm);

// Read `bytes` of `buf` (a buffer larger than L2) so that L2 holds only clean
// lines of it afterwards: a cold cache for the next kernel, without the dirty
// write-back a memset would leave behind (defined in gemv.cu).
cudaError_t launch_l2_flush(const void* buf, size_t bytes, int num_sms, cudaStream_t st);

// One read of `bytes` (a multiple of 16, 16-byte aligned) of `buf` with 16-byte
// streaming loads and nothing else: the HBM read ceiling the GEMVs are held to
// (defined in gemv.cu).
cudaError_t launch_read_probe(const void* buf, size_t bytes, int num_sms, cudaStream_t st);

// Record a message for gemm_last_error() (defined in api.cu).
void set_last_error(const char* msg);

// ---- quantisers (quant.cu): GEMM_Q_* formats of the public header ------------------
cudaError_t launch_quant(int format, const float* src, void* dst, void* scales, long rows, long cols,
                         int num_sms, cudaStream_t st);

// ---- peak probe -----------------------------------------------------------------
cudaError_t launch_peak(int kind, int reps, int ctas, float* sink, int* dev_err,
                        cudaStream_t st);
double peak_flops_per_launch(int kind, int reps, int ctas);

}  // namespace mlpg
