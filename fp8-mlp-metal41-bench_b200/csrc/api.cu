// api.cu -- the extern "C" boundary of libgemm.so (declared in include/mlpgemm.h).
//
// Host-side replacement for the reference's Swift host loop around its
// Metal kernels (main.swift:85-154 dtype/tile tables, :214-244 library
// loading, :486-557 dispatch and timing).  No allocation happens inside
// gemm_run / gemm_time; buffers and workspaces belong to the caller.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

// The library is built with -fvisibility=hidden; only the C ABI is exported.
#pragma GCC visibility push(default)
#include "../../include/mlpgemm.h"
#pragma GCC visibility pop
#include "formats.cuh"
#include "kernels.h"

using namespace mlpg;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(GEMM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

constexpr int kMaxDevices = 16;

struct DevState {
  bool ready = false;
  int* dev_err = nullptr;   // device error word for bounded-wait timeouts
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  char name[256] = {0};
};

DevState g_dev[kMaxDevices];
std::mutex g_mu;

// ---- dtype table (main.swift:85-111) -------------------------------------------
const char* kDtypeNames[kNumDTypes] = {"fp16", "int8", "i8i8", "fp8", "f8f8",
                                        "f4f4", "mxfp4", "mxfp4/a4", "mxfp4/a8", "mxfp4/f8"};
const char* kKernelNames[kNumDTypes] = {"fp16_mlp_gemm", "int8_mlp_gemm", "i8i8_mlp_gemm",
                                         "fp8_mlp_gemm",  "f8f8_mlp_gemm", "f4f4_mlp_gemm",
                                         "mxfp4_mlp_gemm", "mx4x4_mlp_gemm", "mx8x4_mlp_gemm",
                                         "f8x4_mlp_gemm"};

// ---- tile table -----------------------------------------------------------------
enum TileKind { kTileTC = 0, kTileGemv = 1, kTileStream = 2, kTileThin = 3, kTileMma = 4 };
struct TileDef {
  const char* name;
  TileKind kind;
  int param;   // BN for tensor-core tiles, K splits for GEMV tiles
  int bm;      // tensor-core tiles: 128 (one CTA) or 256 (a CTA pair)
};
const TileDef kTiles[] = {
    {"256x256", kTileTC, 256, 256},  {"128x256", kTileTC, 256, 128}, {"128x128", kTileTC, 128, 128},
    {"256x192", kTileTC, 192, 256},
    {"16x128", kTileThin, 0, 0},     {"stream", kTileStream, 0, 0},
    {"gemv.k1", kTileGemv, 1, 0},    {"gemv.k2", kTileGemv, 2, 0},   {"gemv.k4", kTileGemv, 4, 0},
    {"gemv.k8", kTileGemv, 8, 0},    {"gemv.k16", kTileGemv, 16, 0}, {"gemv.k32", kTileGemv, 32, 0},
    {"gemv.k64", kTileGemv, 64, 0},  {"gemv.mma", kTileMma, 0, 0},
    {"256x224", kTileTC, 224, 256},
};
constexpr int kNumTiles = (int)(sizeof(kTiles) / sizeof(kTiles[0]));

bool valid_dtype(int dt) { return dt >= 0 && dt < kNumDTypes; }
bool valid_tile(int t) { return t >= 0 && t < kNumTiles; }

int layout_check(int dt, long N, long K, long M) {
  if (!valid_dtype(dt)) return GEMM_ERR_ARGS;
  if (N <= 0 || K <= 0 || M <= 0) return GEMM_ERR_ARGS;
  const bool fp4ok = ((N * K) % 2 == 0) && ((K * M) % 2 == 0);
  const bool mxok = fp4ok && (K % 32 == 0);
  if (dt == kF4F4 && !fp4ok) return GEMM_ERR_ARGS;
  if ((dt == kMXFP4 || dt == kMX4X4) && !mxok) return GEMM_ERR_ARGS;
  if ((dt == kMX8X4 || dt == kF8X4) && (!mxok || K % 128 != 0)) return GEMM_ERR_ARGS;
  return GEMM_OK;
}

bool any_tc(int dt, int N, int K, int M) {
  for (int t = 0; t < kNumTiles; ++t)
    if (kTiles[t].kind == kTileTC && tc_supported(dt, kTiles[t].bm, kTiles[t].param, N, K, M)) return true;
  return false;
}

bool tile_ok(int dt, int t, int N, int K, int M) {
  if (!valid_tile(t) || layout_check(dt, N, K, M) != GEMM_OK) return false;
  if (kTiles[t].kind == kTileTC) return tc_supported(dt, kTiles[t].bm, kTiles[t].param, N, K, M);
  if (kTiles[t].kind == kTileStream) return stream_supported(dt, N, K, M);
  if (kTiles[t].kind == kTileThin) return thin_supported(dt, N, K, M);
  if (kTiles[t].kind == kTileMma) return mma_supported(dt, N, K, M);
  // CUDA-core tiles: the thin-row kernel, and the fallback where no
  // tensor-core tile covers the dtype or shape.
  if (!gemv_supported(dt, kTiles[t].param, N, K, M)) return false;
  return N <= 16 || !any_tc(dt, N, K, M);
}

DevState* dev_state(int device) {
  if (device < 0 || device >= kMaxDevices) return nullptr;
  DevState* s = &g_dev[device];
  return s->ready ? s : nullptr;
}

int check_dev_error(DevState* s, int device) {
  int h = 0;
  cudaError_t e = cudaMemcpy(&h, s->dev_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (h != 0) {
    cudaMemset(s->dev_err, 0, sizeof(int));
    return fail(GEMM_ERR_TIMEOUT, "device %d: bounded wait expired in a kernel (code %d, site 0x%x)",
                device, h >> 16, h & 0xFFFF);
  }
  return GEMM_OK;
}

int enqueue(DevState* s, int dt, int tile, const void* X, const void* W, void* Y, int N, int K,
            int M, const void* xscale, const void* wscale, void* ws, size_t ws_bytes,
            cudaStream_t st, void* const* ypeers = nullptr, int npeers = 0) {
  RunArgs a;
  a.ypeers = ypeers;
  a.npeers = npeers;
  a.dt = dt;
  a.X = X;
  a.W = W;
  a.Y = Y;
  a.xscale = static_cast<const uint8_t*>(xscale);
  a.wscale = static_cast<const uint8_t*>(wscale);
  a.N = N;
  a.K = K;
  a.M = M;
  a.ws = ws;
  a.ws_bytes = ws_bytes;
  a.stream = st;
  a.dev_err = s->dev_err;
  a.num_sms = s->num_sms;
  cudaError_t e;
  if (kTiles[tile].kind == kTileTC) e = launch_tc(a, kTiles[tile].bm, kTiles[tile].param);
  else if (kTiles[tile].kind == kTileStream) e = launch_stream(a);
  else if (kTiles[tile].kind == kTileThin) e = launch_thin(a);
  else if (kTiles[tile].kind == kTileMma) e = launch_mma(a);
  else e = launch_gemv(a, kTiles[tile].param);
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return GEMM_OK;
}

int validate(int device, int dt, int tile, const void* X, const void* W, void* Y, int N, int K,
             int M, const void* xscale, const void* wscale, void* ws, size_t ws_bytes) {
  if (!valid_dtype(dt)) return fail(GEMM_ERR_ARGS, "unknown dtype %d", dt);
  if (!valid_tile(tile)) return fail(GEMM_ERR_ARGS, "unknown tile %d", tile);
  if (layout_check(dt, N, K, M) != GEMM_OK)
    return fail(GEMM_ERR_ARGS,
                "%s needs N, K, M > 0, even X/W counts and K a multiple of 32 (128 for FP8 x MXFP4)",
                kDtypeNames[dt]);
  if (!tile_ok(dt, tile, N, K, M))
    return fail(GEMM_ERR_ARGS, "tile %s does not support %s at N=%d K=%d M=%d", kTiles[tile].name,
                kDtypeNames[dt], N, K, M);
  if (!X || !W || !Y) return fail(GEMM_ERR_ARGS, "null operand");
  if (x_scaled(dt) && !xscale) return fail(GEMM_ERR_ARGS, "%s needs an X scale plane", kDtypeNames[dt]);
  if (w_is_mx(dt) && !wscale) return fail(GEMM_ERR_ARGS, "%s needs a W scale plane", kDtypeNames[dt]);
  const size_t need = gemm_workspace_size(dt, tile, N, K, M);
  if (need && (!ws || ws_bytes < need))
    return fail(GEMM_ERR_ARGS, "workspace of %zu bytes required", need);
  (void)device;
  return GEMM_OK;
}

}  // namespace

void mlpg::set_last_error(const char* msg) { g_err = msg ? msg : ""; }

extern "C" {

const char* gemm_version(void) { return "mlpgemm 0.1 (sm_100a tcgen05)"; }

const char* gemm_last_error(void) { return g_err.c_str(); }

int gemm_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

int gemm_init(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (device < 0 || device >= kMaxDevices) return fail(GEMM_ERR_INIT, "bad device %d", device);
  DevState* s = &g_dev[device];
  if (s->ready) return GEMM_OK;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n <= device)
    return fail(GEMM_ERR_INIT, "no CUDA device %d (%s)", device,
                e == cudaSuccess ? "not present" : cudaGetErrorString(e));
  cudaDeviceProp prop;
  if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return cuda_fail(e, "device properties");
  if (prop.major != 10 || prop.minor != 0)
    return fail(GEMM_ERR_INIT, "device %d (%s) is sm_%d%d; this library is built for sm_100a", device,
                prop.name, prop.major, prop.minor);
  if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  if ((e = cudaMalloc(&s->dev_err, sizeof(int))) != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  if ((e = cudaMemset(s->dev_err, 0, sizeof(int))) != cudaSuccess) return cuda_fail(e, "cudaMemset");
  if ((e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_fail(e, "cudaStreamCreate");
  s->num_sms = prop.multiProcessorCount;
  snprintf(s->name, sizeof s->name, "%s", prop.name);
  s->ready = true;
  return GEMM_OK;
}

int gemm_device_info(int device, char* name, int name_len, char* arch, int arch_len, int* sm_count) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "device properties");
  if (name && name_len > 0) snprintf(name, name_len, "%s", prop.name);
  if (arch && arch_len > 0) snprintf(arch, arch_len, "sm_%d%d", prop.major, prop.minor);
  if (sm_count) *sm_count = prop.multiProcessorCount;
  return GEMM_OK;
}

const char* gemm_dtype_name(int dtype) { return valid_dtype(dtype) ? kDtypeNames[dtype] : ""; }
const char* gemm_kernel_name(int dtype) { return valid_dtype(dtype) ? kKernelNames[dtype] : ""; }

int gemm_num_tiles(void) { return kNumTiles; }
const char* gemm_tile_name(int tile) { return valid_tile(tile) ? kTiles[tile].name : ""; }
int gemm_tile_index(const char* name) {
  if (!name) return -1;
  for (int t = 0; t < kNumTiles; ++t)
    if (strcmp(kTiles[t].name, name) == 0) return t;
  return -1;
}

int gemm_tile_supported(int dtype, int tile, int N, int K, int M) {
  return tile_ok(dtype, tile, N, K, M) ? 1 : 0;
}

int gemm_check_layout(int dtype, int N, int K, int M) {
  if (layout_check(dtype, N, K, M) != GEMM_OK)
    return fail(GEMM_ERR_ARGS, "layout rule violated for dtype %d at N=%d K=%d M=%d", dtype, N, K, M);
  return GEMM_OK;
}

int gemm_default_tile(int dtype, int N, int K, int M) {
  if (layout_check(dtype, N, K, M) != GEMM_OK) return -1;
  if (N > 16) {
    // block-scaled kinds: the CTA pair (TMA-store epilogue) measures 2-5 % ahead
    // of the 1-CTA 128x256 tile from N = 256 on; below that the pair's second
    // CTA would hold no rows
    const bool scaled = dtype == kMX4X4 || dtype == kMX8X4 || dtype == kF8X4;
    if (scaled && N < 256 && tc_supported(dtype, 128, 256, N, K, M)) return gemm_tile_index("128x256");
    // A16 kinds on the pair tile widen all of W to f16 first: worth it once the
    // per-128-row conversions of the 1-CTA tiles would repeat (N >= 256)
    const bool a16 = dtype == kINT8 || dtype == kFP8 || dtype == kMXFP4;
    // f4f4 (kind::mxf4, unit scale cells copied once), mxfp4/f8 (unit X
    // cells) and mxfp4/a4 (a six-stage ring there): the two accumulators of
    // 256x224 measure ahead of the one of 256x256 (f4f4 fat 70.7 against
    // 74.8 us, square 50.2 against 54.3; mxfp4/f8 0.5-2.7 %; a4 fat 68.8
    // against 70.8 us, square even); a8 is slower there
    if ((dtype == kF4F4 || dtype == kF8X4 || dtype == kMX4X4) && N >= 256 &&
        tc_supported(dtype, 256, 224, N, K, M))
      return gemm_tile_index("256x224");
    if ((!a16 || N >= 256) && tc_supported(dtype, 256, 256, N, K, M)) return gemm_tile_index("256x256");
    if (tc_supported(dtype, 128, 256, N, K, M)) return gemm_tile_index("128x256");
    if (tc_supported(dtype, 128, 128, N, K, M)) return gemm_tile_index("128x128");
  }
  // 3 <= N <= 16: the tensor-core thin tile (weights as the MMA's A operand)
  // measures 1.1-3.6x ahead of the CUDA-core kernels; at N <= 2 the split-K
  // GEMV streams the weights faster
  if (N >= 3 && thin_supported(dtype, N, K, M)) return gemm_tile_index("16x128");
  // MX weights with E2M1 / E4M3 activations (a4, a8, f8) have no 16x128 form;
  // the warp-MMA thin tile runs them 1.8-3.6x faster than the CUDA-core
  // kernel from N = 3 on (N = 4..16, K = 4096, M = 11008)
  const bool mx_q = dtype == kMX4X4 || dtype == kMX8X4 || dtype == kF8X4;
  if (mx_q && N >= 3 && mma_supported(dtype, N, K, M)) return gemm_tile_index("gemv.mma");
  int sms = 148;
  for (int d = 0; d < kMaxDevices; ++d)
    if (g_dev[d].ready) { sms = g_dev[d].num_sms; break; }
  const int s = gemv_auto_ksplit(dtype, N, K, M, sms);
  char name[32];
  snprintf(name, sizeof name, "gemv.k%d", s);
  return gemm_tile_index(name);
}

size_t gemm_workspace_size(int dtype, int tile, int N, int K, int M) {
  if (!valid_tile(tile) || !valid_dtype(dtype)) return 0;
  if (kTiles[tile].kind == kTileTC) return tc_workspace(dtype, kTiles[tile].bm, kTiles[tile].param, N, K, M);
  if (kTiles[tile].kind == kTileStream) return stream_supported(dtype, N, K, M) ? stream_workspace(dtype, N, K, M) : 0;
  if (kTiles[tile].kind == kTileThin) return thin_workspace(dtype, N, K, M);
  if (kTiles[tile].kind == kTileMma) return mma_supported(dtype, N, K, M) ? mma_workspace(dtype, N, K, M) : 0;
  return gemv_workspace(dtype, kTiles[tile].param, N, K, M);
}

int gemm_launches_per_run(int dtype, int tile, int N, int K, int M) {
  (void)N; (void)K; (void)M;
  if (!valid_tile(tile)) return 0;
  return kTiles[tile].kind == kTileTC ? tc_launches(dtype, kTiles[tile].bm) : 1;
}

void* gemm_alloc(int device, size_t bytes) {
  if (cudaSetDevice(device) != cudaSuccess) return nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes ? bytes : 1);
  if (e != cudaSuccess) {
    cuda_fail(e, "cudaMalloc");
    return nullptr;
  }
  return p;
}

int gemm_free(int device, void* ptr) {
  if (cudaSetDevice(device) != cudaSuccess) return fail(GEMM_ERR_CUDA, "cudaSetDevice");
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? GEMM_OK : cuda_fail(e, "cudaFree");
}

int gemm_memset(int device, void* ptr, int value, size_t bytes) {
  if (cudaSetDevice(device) != cudaSuccess) return fail(GEMM_ERR_CUDA, "cudaSetDevice");
  cudaError_t e = cudaMemset(ptr, value, bytes);
  return e == cudaSuccess ? GEMM_OK : cuda_fail(e, "cudaMemset");
}

int gemm_h2d(int device, void* dst, const void* src, size_t bytes) {
  if (cudaSetDevice(device) != cudaSuccess) return fail(GEMM_ERR_CUDA, "cudaSetDevice");
  cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
  return e == cudaSuccess ? GEMM_OK : cuda_fail(e, "cudaMemcpy H2D");
}

int gemm_d2h(int device, void* dst, const void* src, size_t bytes) {
  if (cudaSetDevice(device) != cudaSuccess) return fail(GEMM_ERR_CUDA, "cudaSetDevice");
  cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? GEMM_OK : cuda_fail(e, "cudaMemcpy D2H");
}

void* gemm_host_alloc(size_t bytes) {
  void* p = nullptr;
  if (cudaMallocHost(&p, bytes ? bytes : 1) != cudaSuccess) return nullptr;
  return p;
}

int gemm_host_free(void* ptr) {
  cudaError_t e = cudaFreeHost(ptr);
  return e == cudaSuccess ? GEMM_OK : cuda_fail(e, "cudaFreeHost");
}

int gemm_run(int device, int dtype, int tile, const void* X, const void* W, void* Y, int N, int K,
             int M, const void* xscale, const void* wscale, void* workspace, size_t workspace_bytes,
             void* stream) {
  DevState* s = dev_state(device);
  if (!s) return fail(GEMM_ERR_INIT, "device %d not initialised (call gemm_init)", device);
  int rc = validate(device, dtype, tile, X, W, Y, N, K, M, xscale, wscale, workspace, workspace_bytes);
  if (rc) return rc;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  return enqueue(s, dtype, tile, X, W, Y, N, K, M, xscale, wscale, workspace, workspace_bytes,
                 static_cast<cudaStream_t>(stream));
}

int gemm_run_gather(int device, int dtype, int tile, const void* X, const void* W, void* Y, int N, int K,
                    int M, const void* xscale, const void* wscale, void* workspace, size_t workspace_bytes,
                    void* const* ypeers, int npeers, void* stream) {
  DevState* s = dev_state(device);
  if (!s) return fail(GEMM_ERR_INIT, "device %d not initialised (call gemm_init)", device);
  int rc = validate(device, dtype, tile, X, W, Y, N, K, M, xscale, wscale, workspace, workspace_bytes);
  if (rc) return rc;
  if (npeers < 0 || npeers > GEMM_MAX_PEERS) return fail(GEMM_ERR_ARGS, "npeers %d not in 0..%d", npeers, GEMM_MAX_PEERS);
  if (npeers && !ypeers) return fail(GEMM_ERR_ARGS, "null peer list");
  for (int i = 0; i < npeers; ++i)
    if (!ypeers[i] || (reinterpret_cast<uintptr_t>(ypeers[i]) & 15u))
      return fail(GEMM_ERR_ARGS, "peer Y %d is null or not 16-byte aligned", i);
  if (npeers && (kTiles[tile].kind != kTileTC || !tc_gather_supported(dtype, kTiles[tile].bm)))
    return fail(GEMM_ERR_ARGS, "tile %s has no fused all-gather for %s", kTiles[tile].name, kDtypeNames[dtype]);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  return enqueue(s, dtype, tile, X, W, Y, N, K, M, xscale, wscale, workspace, workspace_bytes,
                 static_cast<cudaStream_t>(stream), ypeers, npeers);
}

int gemm_gather_supported(int dtype, int tile) {
  return valid_dtype(dtype) && valid_tile(tile) && kTiles[tile].kind == kTileTC &&
         tc_gather_supported(dtype, kTiles[tile].bm);
}

int gemm_peer_alloc(int device, size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle) return fail(GEMM_ERR_ARGS, "null output");
  *ptr = nullptr;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaMalloc(ptr, bytes ? bytes : 1);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (peer buffer)");
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_fail(e, "cudaIpcGetMemHandle");
  }
  static_assert(sizeof(h) == GEMM_PEER_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return GEMM_OK;
}

int gemm_peer_open(int device, const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(GEMM_ERR_ARGS, "null argument");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? GEMM_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int gemm_peer_close(int device, void* ptr) {
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? GEMM_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int gemm_sync(int device, void* stream) {
  DevState* s = dev_state(device);
  if (!s) return fail(GEMM_ERR_INIT, "device %d not initialised", device);
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
  return check_dev_error(s, device);
}

int gemm_time(int device, int dtype, int tile, const void* X, const void* const* Ws, void* Y, int N,
              int K, int M, const void* xscale, const void* const* wscales, int nrot, void* workspace,
              size_t workspace_bytes, int warmup, int iters, void* flush, size_t flush_bytes,
              float* ms_out) {
  DevState* s = dev_state(device);
  if (!s) return fail(GEMM_ERR_INIT, "device %d not initialised", device);
  if (!Ws || nrot < 1 || iters < 1 || warmup < 0 || !ms_out) return fail(GEMM_ERR_ARGS, "bad timing arguments");
  for (int r = 0; r < nrot; ++r) {
    int rc = validate(device, dtype, tile, X, Ws[r], Y, N, K, M, xscale, wscales ? wscales[r] : nullptr,
                      workspace, workspace_bytes);
    if (rc) return rc;
  }
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  cudaStream_t st = s->stream;
  std::vector<cudaEvent_t> ev(2 * (size_t)iters);
  for (auto& x : ev)
    if ((e = cudaEventCreate(&x)) != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
  int rc = GEMM_OK;
  for (int i = 0; i < warmup && rc == GEMM_OK; ++i)
    rc = enqueue(s, dtype, tile, X, Ws[i % nrot], Y, N, K, M, xscale, wscales ? wscales[i % nrot] : nullptr,
                 workspace, workspace_bytes, st);
  for (int i = 0; i < iters && rc == GEMM_OK; ++i) {
    if (flush && flush_bytes) {
      e = launch_l2_flush(flush, flush_bytes, s->num_sms, st);
      if (e != cudaSuccess) { rc = cuda_fail(e, "L2 flush"); break; }
    }
    const int r = (warmup + i) % nrot;
    cudaEventRecord(ev[2 * i], st);
    rc = enqueue(s, dtype, tile, X, Ws[r], Y, N, K, M, xscale, wscales ? wscales[r] : nullptr, workspace,
                 workspace_bytes, st);
    cudaEventRecord(ev[2 * i + 1], st);
  }
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess && rc == GEMM_OK) rc = cuda_fail(e, "timing loop");
  if (rc == GEMM_OK) rc = check_dev_error(s, device);
  for (int i = 0; i < iters && rc == GEMM_OK; ++i) {
    float ms = 0.f;
    if ((e = cudaEventElapsedTime(&ms, ev[2 * i], ev[2 * i + 1])) != cudaSuccess) rc = cuda_fail(e, "event time");
    ms_out[i] = ms;
  }
  for (auto& x : ev) cudaEventDestroy(x);
  return rc;
}

int gemm_time_e2e(int device, int dtype, int tile, const void* hX, void* dX, const void* dW, void* dY,
                  void* hY, int N, int K, int M, const void* hxscale, void* dxscale, const void* dwscale,
                  void* workspace, size_t workspace_bytes, int warmup, int iters, float* ms_out) {
  DevState* s = dev_state(device);
  if (!s) return fail(GEMM_ERR_INIT, "device %d not initialised", device);
  if (!hX || !hY || iters < 1 || warmup < 0 || !ms_out) return fail(GEMM_ERR_ARGS, "bad timing arguments");
  int rc = validate(device, dtype, tile, dX, dW, dY, N, K, M, dxscale, dwscale, workspace, workspace_bytes);
  if (rc) return rc;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  const size_t xb = dtype == kF4F4 || dtype == kMX4X4 ? (size_t)N * K / 2
                    : (x_is_half(dtype) ? (size_t)N * K * 2 : (size_t)N * K);
  const size_t xsb = x_scaled(dtype) ? (size_t)N * (K / 32) : 0;
  const size_t yb = (size_t)N * M * 4;
  cudaStream_t st = s->stream;
  std::vector<cudaEvent_t> ev(2 * (size_t)iters);
  for (auto& x : ev)
    if ((e = cudaEventCreate(&x)) != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
  for (int i = 0; i < warmup + iters && rc == GEMM_OK; ++i) {
    const bool timed = i >= warmup;
    if (timed) cudaEventRecord(ev[2 * (i - warmup)], st);
    cudaMemcpyAsync(dX, hX, xb, cudaMemcpyHostToDevice, st);
    if (xsb) cudaMemcpyAsync(dxscale, hxscale, xsb, cudaMemcpyHostToDevice, st);
    rc = enqueue(s, dtype, tile, dX, dW, dY, N, K, M, dxscale, dwscale, workspace, workspace_bytes, st);
    cudaMemcpyAsync(hY, dY, yb, cudaMemcpyDeviceToHost, st);
    if (timed) cudaEventRecord(ev[2 * (i - warmup) + 1], st);
  }
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess && rc == GEMM_OK) rc = cuda_fail(e, "e2e loop");
  if (rc == GEMM_OK) rc = check_dev_error(s, device);
  for (int i = 0; i < iters && rc == GEMM_OK; ++i) {
    float ms = 0.f;
    if ((e = cudaEventElapsedTime(&ms, ev[2 * i], ev[2 * i + 1])) != cudaSuccess) rc = cuda_fail(e, "event time");
    ms_out[i] = ms;
  }
  for (auto& x : ev) cudaEventDestroy(x);
  return rc;
}

int gemm_time_e2e_pipelined(int device, int dtype, int tile, const void* hX, void* dX0, void* dX1, const void* dW,
                            void* dY0, void* dY1, void* hY, int N, int K, int M, const void* hxscale,
                            void* dxscale0, void* dxscale1, const void* dwscale, void* workspace,
                            size_t workspace_bytes, int warmup, int iters, float* total_ms) {
  DevState* s = dev_state(device);
  if (!s) return fail(GEMM_ERR_INIT, "device %d not initialised", device);
  if (!hX || !hY || !dX1 || !dY1 || iters < 1 || warmup < 0 || !total_ms)
    return fail(GEMM_ERR_ARGS, "bad timing arguments");
  int rc = validate(device, dtype, tile, dX0, dW, dY0, N, K, M, dxscale0, dwscale, workspace, workspace_bytes);
  if (rc) return rc;
  if (x_scaled(dtype) && (!hxscale || !dxscale1)) return fail(GEMM_ERR_ARGS, "%s needs X scale planes", kDtypeNames[dtype]);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  const size_t xb = dtype == kF4F4 || dtype == kMX4X4 ? (size_t)N * K / 2
                    : (x_is_half(dtype) ? (size_t)N * K * 2 : (size_t)N * K);
  const size_t xsb = x_scaled(dtype) ? (size_t)N * (K / 32) : 0;
  const size_t yb = (size_t)N * M * 4;
  void* dX[2] = {dX0, dX1};
  void* dY[2] = {dY0, dY1};
  void* dXS[2] = {dxscale0, dxscale1};
  // copies in, GEMMs, copies out: three streams; events order each buffer set's reuse
  cudaStream_t st = s->stream, sin = nullptr, sout = nullptr;
  cudaEvent_t in_done[2] = {}, gemm_done[2] = {}, out_done[2] = {}, t0 = nullptr, t1 = nullptr;
  bool ok = cudaStreamCreateWithFlags(&sin, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&sout, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreate(&t0) == cudaSuccess && cudaEventCreate(&t1) == cudaSuccess;
  for (int b = 0; b < 2 && ok; ++b)
    ok = cudaEventCreateWithFlags(&in_done[b], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&gemm_done[b], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&out_done[b], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) rc = cuda_fail(cudaGetLastError(), "pipeline streams / events");
  for (int i = 0; i < warmup + iters && rc == GEMM_OK; ++i) {
    const int b = i & 1;
    if (i == warmup) {
      // the warm-up steps' copies out may still be running on `sout`: drain all
      // three streams first, so that the timed window holds the timed steps only
      // (and the fill of the first one)
      cudaStreamSynchronize(sin);
      cudaStreamSynchronize(st);
      cudaStreamSynchronize(sout);
      cudaEventRecord(t0, sin);
    }
    cudaStreamWaitEvent(sin, gemm_done[b], 0);   // step i-2 has consumed this X set
    cudaMemcpyAsync(dX[b], hX, xb, cudaMemcpyHostToDevice, sin);
    if (xsb) cudaMemcpyAsync(dXS[b], hxscale, xsb, cudaMemcpyHostToDevice, sin);
    cudaEventRecord(in_done[b], sin);
    cudaStreamWaitEvent(st, in_done[b], 0);
    cudaStreamWaitEvent(st, out_done[b], 0);     // step i-2 has copied this Y set out
    rc = enqueue(s, dtype, tile, dX[b], dW, dY[b], N, K, M, dXS[b], dwscale, workspace, workspace_bytes, st);
    cudaEventRecord(gemm_done[b], st);
    cudaStreamWaitEvent(sout, gemm_done[b], 0);
    cudaMemcpyAsync(hY, dY[b], yb, cudaMemcpyDeviceToHost, sout);
    cudaEventRecord(out_done[b], sout);
    if (i == warmup + iters - 1) cudaEventRecord(t1, sout);
  }
  if (sin && (e = cudaStreamSynchronize(sin)) != cudaSuccess && rc == GEMM_OK) rc = cuda_fail(e, "pipeline copies in");
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess && rc == GEMM_OK) rc = cuda_fail(e, "pipeline GEMMs");
  if (sout && (e = cudaStreamSynchronize(sout)) != cudaSuccess && rc == GEMM_OK) rc = cuda_fail(e, "pipeline copies out");
  if (rc == GEMM_OK) rc = check_dev_error(s, device);
  if (rc == GEMM_OK && (e = cudaEventElapsedTime(total_ms, t0, t1)) != cudaSuccess) rc = cuda_fail(e, "event time");
  for (int b = 0; b < 2; ++b) {
    if (in_done[b]) cudaEventDestroy(in_done[b]);
    if (gemm_done[b]) cudaEventDestroy(gemm_done[b]);
    if (out_done[b]) cudaEventDestroy(out_done[b]);
  }
  if (t0) cudaEventDestroy(t0);
  if (t1) cudaEventDestroy(t1);
  if (sin) cudaStreamDestroy(sin);
  if (sout) cudaStreamDestroy(sout);
  return rc;
}

int gemm_peak_probe(int device, int kind, int reps, int iters, double* tflops_out) {
  DevState* s = dev_state(device);
  if (!s) return fail(GEMM_ERR_INIT, "device %d not initialised", device);
  if (kind < 0 || kind > 14 || reps < 1 || iters < 1 || !tflops_out) return fail(GEMM_ERR_ARGS, "bad probe arguments");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  const int ctas = kind >= 5 ? (s->num_sms / 2) * 2 : s->num_sms;
  float* sink = nullptr;
  if ((e = cudaMalloc(&sink, sizeof(float) * ctas)) != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  std::vector<cudaEvent_t> ev(2 * (size_t)iters);
  for (auto& x : ev) cudaEventCreate(&x);
  int rc = GEMM_OK;
  // two untimed launches, then `iters` timed ones (tune/peak.swift:73-76)
  for (int i = 0; i < 2 + iters && rc == GEMM_OK; ++i) {
    if (i >= 2) cudaEventRecord(ev[2 * (i - 2)], s->stream);
    e = launch_peak(kind, reps, ctas, sink, s->dev_err, s->stream);
    if (e != cudaSuccess) rc = cuda_fail(e, "peak launch");
    if (i >= 2) cudaEventRecord(ev[2 * (i - 2) + 1], s->stream);
  }
  if ((e = cudaStreamSynchronize(s->stream)) != cudaSuccess && rc == GEMM_OK) rc = cuda_fail(e, "peak sync");
  if (rc == GEMM_OK) rc = check_dev_error(s, device);
  if (rc == GEMM_OK) {
    std::vector<float> ms(iters);
    for (int i = 0; i < iters; ++i) cudaEventElapsedTime(&ms[i], ev[2 * i], ev[2 * i + 1]);
    std::sort(ms.begin(), ms.end());
    const double med = ms[iters / 2] * 1e-3;
    *tflops_out = peak_flops_per_launch(kind, reps, ctas) / med / 1e12;
  }
  for (auto& x : ev) cudaEventDestroy(x);
  cudaFree(sink);
  return rc;
}

int gemm_read_probe(int device, const void* buf, size_t bytes, int warmup, int iters, void* flush,
                    size_t flush_bytes, float* ms_out) {
  DevState* s = dev_state(device);
  if (!s) return fail(GEMM_ERR_INIT, "device %d not initialised", device);
  if (!buf || bytes == 0 || bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(buf) & 15) != 0)
    return fail(GEMM_ERR_ARGS, "read probe: buffer must be 16-byte aligned and bytes a non-zero multiple of 16");
  if (iters < 1 || warmup < 0 || !ms_out) return fail(GEMM_ERR_ARGS, "bad timing arguments");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  cudaStream_t st = s->stream;
  std::vector<cudaEvent_t> ev(2 * (size_t)iters);
  for (auto& x : ev)
    if ((e = cudaEventCreate(&x)) != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
  int rc = GEMM_OK;
  for (int i = 0; i < warmup + iters && rc == GEMM_OK; ++i) {
    const int t = i - warmup;
    if (t >= 0 && flush && flush_bytes) {
      e = launch_l2_flush(flush, flush_bytes, s->num_sms, st);
      if (e != cudaSuccess) { rc = cuda_fail(e, "L2 flush"); break; }
    }
    if (t >= 0) cudaEventRecord(ev[2 * t], st);
    e = launch_read_probe(buf, bytes, s->num_sms, st);
    if (e != cudaSuccess) rc = cuda_fail(e, "read probe launch");
    if (t >= 0) cudaEventRecord(ev[2 * t + 1], st);
  }
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess && rc == GEMM_OK) rc = cuda_fail(e, "read probe");
  for (int i = 0; i < iters && rc == GEMM_OK; ++i) {
    float ms = 0.f;
    if ((e = cudaEventElapsedTime(&ms, ev[2 * i], ev[2 * i + 1])) != cudaSuccess) rc = cuda_fail(e, "event time");
    ms_out[i] = ms;
  }
  for (auto& x : ev) cudaEventDestroy(x);
  return rc;
}

int gemm_quantize(int device, int format, const float* src, void* dst, void* scales, long rows, long cols,
                  void* stream) {
  DevState* s = dev_state(device);
  if (!s) return fail(GEMM_ERR_INIT, "device %d not initialised", device);
  if (format < GEMM_Q_E4M3_REF || format > GEMM_Q_MXFP8) return fail(GEMM_ERR_ARGS, "unknown format %d", format);
  if (rows <= 0 || cols <= 0 || !src || !dst) return fail(GEMM_ERR_ARGS, "bad quantiser arguments");
  const bool mx = format == GEMM_Q_MXFP4 || format == GEMM_Q_MXFP8;
  if (mx && (cols % 32 != 0 || !scales))
    return fail(GEMM_ERR_ARGS, "MX formats need cols %% 32 == 0 and a scale plane");
  if ((format == GEMM_Q_E2M1 || format == GEMM_Q_MXFP4) && (rows * cols) % 2 != 0)
    return fail(GEMM_ERR_ARGS, "E2M1 packs two per byte: rows*cols must be even");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : s->stream;
  e = launch_quant(format, src, dst, scales, rows, cols, s->num_sms, st);
  if (e != cudaSuccess) return cuda_fail(e, "quantiser launch");
  return GEMM_OK;
}

}  // extern "C"
