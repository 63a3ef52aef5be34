// noalloc.cu -- gemm_run_noalloc: the thin-row split-K GEMM without any
// caller-provided or library-allocated workspace.
//
// Some callers hand this library nothing but their input and output
// buffers: plugin hosts and serving loops that own every device allocation
// and forbid new ones once they are running, and language bindings that
// expose no allocator.  They cannot call cudaMalloc, and they cannot supply
// the split-K workspace that gemm_run asks for.  For them this file keeps
// the workspace in a fixed device array that is part of the loaded library.
//
// Limits and rules:
//   * capacity: kNoAllocBytes (8 MiB) per GPU, held from the moment the
//     library's device code is loaded on that GPU until the process exits.
//     The first 64 KiB are the split-K tile counters, the rest the partial
//     sums (ksplit * N * M four-byte values).  Larger requests are rejected
//     with GEMM_ERR_ARGS.
//   * the array's host-side name is only a stand-in: its device address is
//     looked up once per device with cudaGetSymbolAddress, with that device
//     current, on the first call for that device.  Make that first call
//     before any stream capture.
//   * every call shares the one array, and it keeps whatever the previous
//     call left there.  Each call clears the counters it uses (an async
//     memset on the caller's stream) before its kernel.  Calls that overlap
//     on the GPU (different streams, no ordering between them) race on the
//     array and give wrong results: serialise them.
//   * no cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#pragma GCC visibility push(default)
#include "../../include/mlpgemm.h"
#pragma GCC visibility pop
#include "formats.cuh"
#include "kernels.h"

using namespace mlpg;

namespace {

constexpr size_t kNoAllocBytes = 8u << 20;       // the stated maximum
constexpr size_t kCounterRegion = 64u << 10;     // split-K tile counters (fixed offset)

// The scratch array.  In host code this name is a host-side shadow, not a
// device address; only the address from cudaGetSymbolAddress may be passed
// to a kernel.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDev = 16;
void* g_scratch_ptr[kMaxDev] = {nullptr};
std::mutex g_scratch_mu;
int err(int code, const std::string& m) {
  set_last_error(("gemm_run_noalloc: " + m).c_str());   // read back with gemm_last_error()
  return code;
}

// One-time, per device: the device address of the scratch array.
int scratch_for(int device, void** out) {
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return err(GEMM_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  return GEMM_OK;
}

}  // namespace

extern "C" int gemm_run_noalloc(int device, int dtype, int ksplit, const void* X, const void* W,
                                void* Y, int N, int K, int M, const void* xscale,
                                const void* wscale, void* stream) {
  if (device < 0 || device >= kMaxDev) return err(GEMM_ERR_ARGS, "bad device");
  if (dtype < 0 || dtype >= kNumDTypes) return err(GEMM_ERR_ARGS, "unknown dtype");
  if (gemm_check_layout(dtype, N, K, M) != GEMM_OK)
    return err(GEMM_ERR_ARGS, "layout rule violated (see gemm_check_layout)");
  if (N > 16) return err(GEMM_ERR_ARGS, "gemm_run_noalloc serves thin rows only (N <= 16)");
  if (!X || !W || !Y) return err(GEMM_ERR_ARGS, "null operand");
  if (x_scaled(dtype) && !xscale) return err(GEMM_ERR_ARGS, "missing X scale plane");
  if (w_is_mx(dtype) && !wscale) return err(GEMM_ERR_ARGS, "missing W scale plane");
  // the caller's current device is put back on every return path
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  struct Restore {
    int dev;
    ~Restore() {
      if (dev >= 0) cudaSetDevice(dev);
    }
  } restore{prev};
  int rc;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return err(GEMM_ERR_CUDA, cudaGetErrorString(e));
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (ksplit <= 0) ksplit = gemv_auto_ksplit(dtype, N, K, M, sms);
  if (!gemv_supported(dtype, ksplit, N, K, M)) {
    char m[256];
    snprintf(m, sizeof m,
             "ksplit=%d is not available for this dtype and shape (N=%d, K=%d, M=%d):"
             " a split must fit the kernel's shared-memory budget, and above 8 splits the output's"
             " tile count must fit the split-K counter region",
             ksplit, N, K, M);
    return err(GEMM_ERR_ARGS, m);
  }
  const size_t need = gemv_workspace(dtype, ksplit, N, K, M);
  if (need > kNoAllocBytes) {
    char m[256];
    snprintf(m, sizeof m,
             "split-K scratch of %zu bytes (ksplit=%d, N=%d, M=%d) exceeds the fixed %zu-byte array;"
             " use a smaller ksplit or gemm_run with a workspace",
             need, ksplit, N, M, kNoAllocBytes);
    return err(GEMM_ERR_ARGS, m);
  }
  void* scratch = nullptr;
  if ((rc = scratch_for(device, &scratch)) != GEMM_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (need) {
    e = cudaMemsetAsync(scratch, 0, kCounterRegion, st);   // counters start at zero
    if (e != cudaSuccess) return err(GEMM_ERR_CUDA, cudaGetErrorString(e));
  }
  RunArgs a;
  a.dt = dtype;
  a.X = X;
  a.W = W;
  a.Y = Y;
  a.xscale = static_cast<const uint8_t*>(xscale);
  a.wscale = static_cast<const uint8_t*>(wscale);
  a.N = N;
  a.K = K;
  a.M = M;
  a.ws = need ? scratch : nullptr;
  a.ws_bytes = need ? kNoAllocBytes : 0;
  a.stream = st;
  a.dev_err = nullptr;
  a.num_sms = sms;
  e = launch_gemv(a, ksplit);
  if (e != cudaSuccess) return err(GEMM_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e));
  return GEMM_OK;
}
