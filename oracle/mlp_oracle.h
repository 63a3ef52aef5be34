/*
 * mlp_oracle.h -- CPU oracle for the MLP GEMM  Y[N,M] = X[N,K] @ W[K,M].
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library; the
 * product (libgemm.so and the mlpgemm package) never links or calls it.
 *
 * This is a plain-C restatement of the reference's CPU-side semantics for
 * the hot path (Anemll/fp8-mlp-metal41-bench):
 *   - number formats            main.swift:4-83
 *   - operand decode semantics  main.swift:419-449 (refActivation/refWeight)
 *   - sample points             main.swift:452-466
 *   - the reference check       main.swift:560-594 (f32 K-order dot product,
 *                               int32 dot product for i8i8)
 *   - the E2M1->E4M3 widening   fp8_mlp.metal:305-309
 * plus an fp64 / int64 dot product (the tighter parity target) and a
 * multithreaded f32 host GEMM that re-runs the reference's CPU dot product
 * over the whole output (the timed CPU baseline).
 *
 * Parity pinning: the reference ships no golden vectors and its Metal/Swift
 * code cannot run on Linux.  The decoders are pinned against constant
 * tables read out of the reference sources (tests/golden/), and the host
 * check semantics are restated line by line; the GEMM arithmetic itself has
 * no reference outputs to compare with.
 */
#ifndef MLP_ORACLE_H
#define MLP_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes: the order of `enum DType` (main.swift:85-95). */
enum {
    ORC_FP16 = 0, ORC_INT8 = 1, ORC_I8I8 = 2, ORC_FP8 = 3, ORC_F8F8 = 4,
    ORC_F4F4 = 5, ORC_MXFP4 = 6, ORC_MX4X4 = 7, ORC_MX8X4 = 8, ORC_F8X4 = 9,
    ORC_NUM_DTYPES = 10
};

/* ---- scalar formats (main.swift:4-83) ---------------------------------- */
uint16_t orc_f32_to_f16(float x);             /* Swift Float16(x): RNE        */
float    orc_f16_to_f32(uint16_t h);
uint8_t  orc_f32_to_e4m3_ref(float x);        /* floatToE4M3, main.swift:6-27 */
uint8_t  orc_f32_to_e4m3_rne(float x);        /* OCP E4M3FN, RNE, satfinite   */
float    orc_e4m3_to_f32(uint8_t b);          /* e4m3ToFloat, main.swift:30-41*/
float    orc_e2m1_to_f32(uint8_t nibble);     /* e2m1ToFloat, main.swift:44-48*/
uint8_t  orc_e2m1_code(long i);               /* e2m1Code,    main.swift:50-53*/
float    orc_e2m1_at(const uint8_t *packed, long index); /* main.swift:69-73 */
float    orc_ue8m0_to_f32(uint8_t code);      /* main.swift:76-78             */
uint8_t  orc_ue8m0_code(long i);              /* main.swift:80-83             */
uint8_t  orc_e2m1_to_e4m3_byte(uint8_t nibble); /* fp8_mlp.metal:305-309 LUT  */
void     orc_pack_e2m1(const uint8_t *codes, long count, uint8_t *out); /* :56-67 */

/* ---- quantisers (the wire formats produced from f32) ----------------------
 * E4M3: orc_f32_to_e4m3_ref / _rne above.  E2M1: OCP round to nearest even on
 * {0, .5, 1, 1.5, 2, 3, 4, 6}, saturating at +-6, sign kept (also for -0);
 * NaN -> 0x7.  MX (OCP MX v1.0 block scaling), one UE8M0 scale per 32
 * consecutive elements of a row: X = floor(log2(amax)) - emax (emax 2 for
 * E2M1, 8 for E4M3) clamped to [-127, 127], scale code X + 127, elements
 * quantised (RNE, saturating) from v * 2^-X.  amax == 0 gives code 0 and zero
 * elements; a block holding NaN or Inf gets scale code 0xFF (NaN) and zero
 * elements.  elem 0: E2M1 packed two per byte along the row (low nibble =
 * even element, main.swift:56-67); elem 1: one E4M3 byte per element. */
uint8_t  orc_f32_to_e2m1_rne(float x);
int      orc_quantize_mx(int elem, const float *src, long rows, long cols,
                         uint8_t *vals, uint8_t *scales);

/* ---- operand decode (main.swift:419-449) ---------------------------------
 * X: the activation buffer the dtype uses (main.swift:477-483); xscale is the
 * [N, K/32] UE8M0 plane (mxfp4/a4, mxfp4/a8 only, else NULL).
 * W: the weight buffer (main.swift:408-418); [K,M] row-major except the MX
 * family, which stores W as [M,K] (main.swift:374-375) with wscale [M, K/32].
 * Decoded X is written [N*K] (row-major), decoded W as [K*M] (w[k*M+m]).
 * Returns 0, or 1 on a layout violation (odd FP4 count, K%32, K%128). */
int orc_decode_x(int dtype, const void *X, const uint8_t *xscale,
                 long N, long K, double *out);
int orc_decode_w(int dtype, const void *W, const uint8_t *wscale,
                 long K, long M, double *out);
int orc_check_layout(int dtype, long N, long K, long M);

/* ---- dot products on decoded operands ------------------------------------
 * Each evaluates `count` outputs (rows[i], cols[i]) of Y.  xd/wd are the
 * decoded operands from orc_decode_x / orc_decode_w. */
void orc_dot_f64(const double *xd, const double *wd, long K, long M,
                 const long *rows, const long *cols, long count, double *out);
/* i8i8: exact int64 dot product on the raw int8 operands (main.swift:563-568). */
void orc_dot_i64(const int8_t *X, const int8_t *W, long K, long M,
                 const long *rows, const long *cols, long count, int64_t *out);
/* The reference's own f32 check: acc += x*w in K order, single precision
 * (main.swift:577-583). */
void orc_dot_f32_korder(const double *xd, const double *wd, long K, long M,
                        const long *rows, const long *cols, long count,
                        float *out);

/* Sample points (main.swift:452-466): tile corners and the far corner,
 * clipped and de-duplicated.  Writes up to 6 points; returns the count. */
int orc_sample_points(long N, long M, int bm, int bn, long *rows, long *cols);

/* ---- multithreaded host GEMM (CPU baseline) -------------------------------
 * The reference's CPU dot product (main.swift:577-583) run over rows
 * [row0, row0+nrows) of the whole output: operands pre-decoded to f32,
 * f32 multiply then add, in K order, one accumulator per output, OpenMP over
 * (row, column block).  Y is [nrows, M].  nthreads<=0 uses all cores. */
void orc_host_gemm_f32(const float *xf, const float *wf, long K, long M,
                       long row0, long nrows, float *Y, int nthreads);
/* i8i8: int32 accumulation (main.swift:563-568). */
void orc_host_gemm_i32(const int8_t *X, const int8_t *W, long K, long M,
                       long row0, long nrows, int32_t *Y, int nthreads);
int  orc_num_threads(void);

/* The reference's deterministic operand patterns (main.swift:364-390):
 * X = (i%97-48)*0.02, W = (i%53-26)*0.05, FP4 code cycles with offsets
 * 0 / +3 / +5, UE8M0 cycles with offsets 0 (W) / +1 (X).  NULL skips. */
void orc_ref_operands(long N, long K, long M,
                      uint16_t *x_f16, int8_t *x_i8, uint8_t *x_e4m3, uint8_t *x_fp4,
                      uint16_t *w_f16, int8_t *w_i8, uint8_t *w_e4m3, uint8_t *w_fp4,
                      uint8_t *w_mx, uint8_t *wscale, uint8_t *xscale);

#ifdef __cplusplus
}
#endif
#endif
