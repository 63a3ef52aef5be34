/*
 * mlpgemm.h -- C ABI of libgemm.so, the B200 (sm_100a) MLP GEMM library.
 *
 *     Y[N,M] = X[N,K] @ W[K,M]          (row-major, caller-owned buffers)
 *
 * The reference (Anemll/fp8-mlp-metal41-bench) exposes this GEMM as Metal
 * compute kernels named "<kernel>_<BM>x<BN>" with buffer slots X@0, W@1,
 * Y@2, N@3, K@4, M@5 and the UE8M0 scale planes at @6/@7, dispatched one
 * command buffer at a time by the Swift host (fp8_mlp.metal:114-461,
 * main.swift:486-521).  Each entry point below says which part of that
 * interface it replaces.  Plain pointers and sizes only; no C++ or torch
 * types cross this boundary.
 *
 * Operand layouts (identical to the reference's buffers, main.swift:364-418):
 *   X      fp16 | int8 | fp8 | mxfp4 : IEEE half [N,K]
 *          i8i8                        : int8 [N,K]
 *          f8f8 | mxfp4/a8 | mxfp4/f8  : E4M3 bytes [N,K]
 *          f4f4 | mxfp4/a4             : E2M1, two per byte along K, low nibble = even element
 *   W      fp16 half [K,M]; int8/i8i8 int8 [K,M]; fp8/f8f8 E4M3 [K,M];
 *          f4f4 E2M1 [K,M] packed along M;
 *          mxfp4, mxfp4/a4, mxfp4/a8, mxfp4/f8: E2M1 stored TRANSPOSED [M,K],
 *          packed along K
 *   xscale UE8M0 [N, K/32]  (mxfp4/a4, mxfp4/a8; slot @6 in the reference)
 *   wscale UE8M0 [M, K/32]  (every mxfp4* dtype; slot @6 or @7)
 *   Y      float32 [N,M]; int32 [N,M] for i8i8.  Y is overwritten.
 * Layout rules (main.swift:473-476): f4f4 needs even N*K and K*M; the mxfp4
 * family needs K % 32 == 0; mxfp4/a8 and mxfp4/f8 need K % 128 == 0.
 *
 * Every function returns a status code (GEMM_OK ... ) unless stated.
 * The library allocates no device memory inside gemm_run / gemm_time:
 * buffers (and the workspace some kernels need) come from the caller.
 */
#ifndef MLPGEMM_H
#define MLPGEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (the reference's exit codes 1/2/3 keep their meaning) -- */
#define GEMM_OK           0
#define GEMM_ERR_ARGS     1  /* bad argument, shape or layout  (main.swift exit(1)) */
#define GEMM_ERR_INIT     2  /* device / library initialisation (exit(2))          */
#define GEMM_ERR_MISMATCH 3  /* result check failed (used by drivers, exit(3))      */
#define GEMM_ERR_CUDA     4  /* CUDA runtime error                                  */
#define GEMM_ERR_TIMEOUT  5  /* a device-side bounded wait expired                  */

/* ---- dtypes: the order of `enum DType`, main.swift:85-95 ------------------ */
#define GEMM_FP16      0
#define GEMM_INT8      1
#define GEMM_I8I8      2
#define GEMM_FP8       3
#define GEMM_F8F8      4
#define GEMM_F4F4      5
#define GEMM_MXFP4     6
#define GEMM_MXFP4_A4  7
#define GEMM_MXFP4_A8  8
#define GEMM_MXFP4_F8  9
#define GEMM_NUM_DTYPES 10

/* ---- library / device ---------------------------------------------------- */

/* Select and initialise a CUDA device, check it is sm_100 and load the
 * kernels.  Replaces MTLCreateSystemDefaultDevice + loadLibrary
 * (main.swift:214-244, :272-297).  Returns GEMM_ERR_INIT if no usable B200. */
int gemm_init(int device);

/* Number of visible CUDA devices (0 on a host without a GPU). */
int gemm_device_count(void);

/* Device name and architecture string ("sm_100"), the inputs of the profile
 * slug (device.name and device.architecture.name, main.swift:320-326). */
int gemm_device_info(int device, char *name, int name_len, char *arch, int arch_len,
                     int *sm_count);

/* Most recent error message of the calling thread ("" if none). */
const char *gemm_last_error(void);

/* Library version string. */
const char *gemm_version(void);

/* ---- dtypes and tiles ---------------------------------------------------- */

/* dtype name as on the reference CLI ("fp16" ... "mxfp4/f8") and its
 * reference kernel name ("fp16_mlp_gemm" ...), main.swift:85-111. */
const char *gemm_dtype_name(int dtype);
const char *gemm_kernel_name(int dtype);

/* The tile list that replaces the reference's ten BMxBN threadgroup tiles
 * (main.swift:135-143, fp8_mlp.metal:446-450).  Tensor-core tiles are named
 * "<BM>x<BN>" (BM rows of Y per CTA, BN columns); the CUDA-core split-K
 * kernels for thin rows are named "gemv.k<S>" (S = K splits); "16x128" is the
 * tcgen05 thin tile, "stream" the persistent streaming GEMV and "gemv.mma" the
 * thin tile on warp-level MMAs (N <= 16; fp16, int8, fp8, f8f8 with K % 4 and
 * 16-byte weight rows, the MX kinds with K % 128). */
int gemm_num_tiles(void);
const char *gemm_tile_name(int tile);
int gemm_tile_index(const char *name);          /* -1 if unknown */

/* 1 if `tile` can run this dtype and shape, else 0. */
int gemm_tile_supported(int dtype, int tile, int N, int K, int M);

/* Built-in default tile (defaultTile, main.swift:148-154). */
int gemm_default_tile(int dtype, int N, int K, int M);

/* Layout rules of main.swift:473-476; GEMM_OK or GEMM_ERR_ARGS. */
int gemm_check_layout(int dtype, int N, int K, int M);

/* Bytes of device workspace gemm_run needs for this dtype/tile/shape
 * (split-K partial sums and counters, the f4f4 weight transpose).  0 means
 * no workspace.  Counters in the workspace must be zero before the first
 * call; every kernel leaves them zero on exit. */
size_t gemm_workspace_size(int dtype, int tile, int N, int K, int M);

/* ---- memory (for callers without their own allocator) -------------------- */
void *gemm_alloc(int device, size_t bytes);
int gemm_free(int device, void *ptr);
int gemm_memset(int device, void *ptr, int value, size_t bytes);
int gemm_h2d(int device, void *dst, const void *src, size_t bytes);
int gemm_d2h(int device, void *dst, const void *src, size_t bytes);
/* Page-locked host memory, for end-to-end copies. */
void *gemm_host_alloc(size_t bytes);
int gemm_host_free(void *ptr);

/* ---- compute --------------------------------------------------------------- */

/* Enqueue one GEMM on `stream` (a cudaStream_t; NULL = the default stream).
 * Replaces one dispatchThreadgroups of "<kernel>_<tile>" with the buffer
 * bindings of main.swift:497-511.  xscale/wscale follow the slot rules of
 * main.swift:505-510 (pass NULL where the dtype has no plane).  `workspace`
 * must hold gemm_workspace_size() bytes (NULL if that is 0).
 * Asynchronous: errors of the kernel itself surface at gemm_sync. */
int gemm_run(int device, int dtype, int tile, const void *X, const void *W, void *Y,
             int N, int K, int M, const void *xscale, const void *wscale,
             void *workspace, size_t workspace_bytes, void *stream);

/* ---- fused GEMM + all-gather over NVLink (multi-GPU; no reference analogue:
 * the reference is single-device, main.swift:272) ------------------------------
 *
 * gemm_run_gather is gemm_run whose tensor-core epilogue also writes every Y
 * element at the same byte offset from each of `npeers` peer pointers: the
 * Y buffers of the other GPUs, mapped into this device with gemm_peer_open.
 * With rows of X split across GPUs and every GPU's block at its own rows
 * of a full-size Y, one call per GPU leaves the whole Y on every GPU: the
 * all-gather happens inside the GEMM, tile by tile, with no collective
 * launch.  The peers' writes into this GPU's Y are complete once every
 * GPU's call has finished on its stream (synchronise the GPUs after the
 * calls, e.g. with a small all-reduce on the same stream).
 * npeers 0 is gemm_run.  Tensor-core tiles only, except the 1-CTA tiles of
 * the A16 kinds (int8, fp8, mxfp4 at 128x256 / 128x128): gemm_gather_supported.
 * Peer pointers must be 16-byte aligned. */
#define GEMM_MAX_PEERS 7
#define GEMM_PEER_HANDLE_BYTES 64
int gemm_run_gather(int device, int dtype, int tile, const void *X, const void *W, void *Y,
                    int N, int K, int M, const void *xscale, const void *wscale,
                    void *workspace, size_t workspace_bytes, void *const *ypeers, int npeers,
                    void *stream);
int gemm_gather_supported(int dtype, int tile);
/* Device memory that other processes can map: *ptr gets the allocation (free
 * it with gemm_free) and `handle` its GEMM_PEER_HANDLE_BYTES-byte IPC handle. */
int gemm_peer_alloc(int device, size_t bytes, void **ptr, void *handle);
/* Map another process's gemm_peer_alloc buffer into `device`; unmap with
 * gemm_peer_close. */
int gemm_peer_open(int device, const void *handle, void **ptr);
int gemm_peer_close(int device, void *ptr);

/* Wait for all work on `stream` and check the device error word (timeouts of
 * bounded waits).  The cb.waitUntilCompleted + status check of
 * main.swift:513-518. */
int gemm_sync(int device, void *stream);

/* Time `iters` GEMMs after `warmup` untimed ones, one CUDA-event pair per
 * iteration on an internal stream, launches queued back to back (the runOnce
 * loop of main.swift:545-555 with GPU timestamps replaced by CUDA events).
 * Ws / wscales are arrays of `nrot` weight copies used round-robin, so that
 * weights smaller than L2 still stream from HBM every iteration (nrot = 1:
 * the reference's behaviour).  If `flush` is non-NULL, `flush_bytes` of it
 * (more than the 126 MB L2) are read before every timed iteration, outside
 * its event pair, so each timed GEMM starts with an L2 holding only clean
 * lines of that buffer.  ms_out receives `iters` times. */
int gemm_time(int device, int dtype, int tile, const void *X, const void *const *Ws, void *Y,
              int N, int K, int M, const void *xscale, const void *const *wscales, int nrot,
              void *workspace, size_t workspace_bytes, int warmup, int iters,
              void *flush, size_t flush_bytes, float *ms_out);

/* Like gemm_time, but each iteration also copies X (and xscale) from pinned
 * host memory before the GEMM and Y back to pinned host memory after it, all
 * inside the timed region (end-to-end time through this C ABI). */
int gemm_time_e2e(int device, int dtype, int tile, const void *hX, void *dX,
                  const void *dW, void *dY, void *hY, int N, int K, int M,
                  const void *hxscale, void *dxscale, const void *dwscale,
                  void *workspace, size_t workspace_bytes, int warmup, int iters,
                  float *ms_out);

/* End-to-end throughput with consecutive steps overlapped.  Each step copies X
 * (and xscale) from pinned host memory in on its own stream, runs the GEMM on
 * the device's stream and copies Y out to pinned host memory on a third stream;
 * two device sets of X / Y are used in turn, so that step i's Y copy overlaps
 * step i+1's X copy and GEMM (the two copy directions run on separate engines).
 * Every step still moves its own inputs in and its own result out.  After
 * `warmup` untimed steps (and once their last copy out has finished), *total_ms
 * receives the time of `iters` steps, from the first timed copy in to the last
 * copy out.  The serving-loop form of runOnce
 * (main.swift:486-518) with the host copies that a plugin host adds. */
int gemm_time_e2e_pipelined(int device, int dtype, int tile, const void *hX, void *dX0, void *dX1,
                            const void *dW, void *dY0, void *dY1, void *hY, int N, int K, int M,
                            const void *hxscale, void *dxscale0, void *dxscale1, const void *dwscale,
                            void *workspace, size_t workspace_bytes, int warmup, int iters,
                            float *total_ms);

/* Per-launch kernel time of the dominant kernel inside gemm_time's loop, and
 * the number of kernels one gemm_run launches (for the roofline report). */
int gemm_launches_per_run(int dtype, int tile, int N, int K, int M);

/* ---- thin rows without any allocation ------------------------------------------
 * No counterpart in the reference (whose Metal host allocates freely).
 * For callers that may not allocate device memory and can only pass their
 * own inputs and outputs: plugin hosts and serving loops that own every
 * device allocation and forbid new ones after start-up, and bindings that
 * expose no allocator.  Same operands, layouts and results as gemm_run with
 * a "gemv.k<ksplit>" tile (N <= 16; ksplit <= 0 picks one), but the split-K
 * scratch lives in a fixed 8 MiB device array inside the library, held on
 * every GPU that loads the library until the process exits.  Requests whose
 * scratch (64 KiB of counters + ksplit*N*M*4 bytes) exceeds 8 MiB return
 * GEMM_ERR_ARGS.  The first call on a device looks up the array's address on
 * that device; make it before any stream capture.  All calls share the array
 * (each clears its counters first): calls that overlap on the GPU race and
 * must be serialised by the caller.  Calls no cudaMalloc / cudaFree.  A split
 * the kernel cannot take (shared memory, or more split-K tiles than the counter
 * region holds) returns GEMM_ERR_ARGS with the reason; the caller's current
 * device is the same on return. */
int gemm_run_noalloc(int device, int dtype, int ksplit, const void *X, const void *W, void *Y,
                     int N, int K, int M, const void *xscale, const void *wscale, void *stream);

/* ---- pure-compute peak probe (tune/peak.metal + tune/peak.swift) ------------ */
/* kind: 0 f16, 1 i8, 2 f8f6f4 (E4M3), 3 mxf8f6f4 (E4M3 x E2M1), 4 mxf4, and
 * 5 f16 / 6 i8 / 7 f8f6f4 on CTA pairs (cta_group::2); 8 f16 / 9 i8 /
 * 10 f8f6f4 on CTA pairs with B read MN-major (the layout of [K,M] weights,
 * as the GEMM's pair tiles read W); 11 mxf8f6f4 / 12 mxf4 on CTA pairs, and
 * 13 / 14 the same with the GEMM's per-stage scale-cell copies (tcgen05.cp)
 * before each stage's MMAs.  Runs 2 untimed and
 * `iters` timed launches of a kernel that issues reps x 4 tcgen05.mma
 * (128 x 256 per CTA, or 256 x 256 per pair) on operands resident in shared
 * memory, no global traffic in the loop (tune/peak.metal:29-87), and
 * reports the median dense TFLOP/s (TOP/s for i8).  The probe allocates a
 * few hundred bytes of device memory for its result sink. */
int gemm_peak_probe(int device, int kind, int reps, int iters, double *tflops_out);

/* Plain streaming read of `bytes` (a non-zero multiple of 16) of the device
 * buffer `buf` (16-byte aligned): coalesced 16-byte loads, eight in flight per
 * thread, one 32 KB run per 256-thread CTA, nothing decoded or written.  The
 * reference has no counterpart; it is the practical HBM ceiling that the
 * thin-row (N <= 16, main.swift:146-150) GEMVs are reported against.  Runs
 * `warmup` untimed launches, then `iters` timed ones on the device's library
 * stream, each preceded (when flush/flush_bytes are given) by a read of the
 * flush buffer so that L2 holds none of `buf`; writes one CUDA-event time (ms)
 * per timed launch to ms_out[0..iters). */
int gemm_read_probe(int device, const void *buf, size_t bytes, int warmup, int iters, void *flush,
                    size_t flush_bytes, float *ms_out);

/* ---- quantisers: the operand formats produced from f32 on the device ---------
 * Replaces the reference's host-side producers, which run untimed before the
 * buffers are made (main.swift:6-27 floatToE4M3, :50-67 E2M1 codes packed two
 * per byte with the low nibble the even element, :76-83 UE8M0 codes).
 * src is f32 [rows, cols] on the device; dst receives:
 *   GEMM_Q_E4M3_REF  one byte per element, floatToE4M3 bit for bit
 *   GEMM_Q_E4M3      one byte per element, OCP E4M3FN round-to-nearest-even
 *                    with subnormals, saturating at +-448, NaN -> 0x7F
 *   GEMM_Q_E2M1      two per byte (rows*cols even), round-to-nearest-even,
 *                    saturating at +-6, NaN -> 0x7
 *   GEMM_Q_MXFP4     OCP MX: E2M1 two per byte plus one UE8M0 code per 32
 *   GEMM_Q_MXFP8     OCP MX: one E4M3 byte per element plus one UE8M0 per 32
 * For the MX formats cols % 32 == 0 and `scales` receives [rows, cols/32]:
 * X = floor(log2(max |v| of the 32)) - emax (2 for E2M1, 8 for E4M3) clamped to
 * [-127, 127], code X + 127, elements quantised from v * 2^-X; a block of
 * zeros gets code 0, a block holding NaN or Inf code 0xFF and zero elements.
 * Asynchronous on `stream` (NULL: the device's library stream). */
#define GEMM_Q_E4M3_REF 0
#define GEMM_Q_E4M3     1
#define GEMM_Q_E2M1     2
#define GEMM_Q_MXFP4    3
#define GEMM_Q_MXFP8    4
int gemm_quantize(int device, int format, const float *src, void *dst, void *scales,
                  long rows, long cols, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* MLPGEMM_H */
