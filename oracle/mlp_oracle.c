/*
 * mlp_oracle.c -- CPU oracle for the MLP GEMM (test infrastructure only).
 *
 * Restates the reference's host-side semantics (Anemll/fp8-mlp-metal41-bench,
 * main.swift) in C.  Nothing in the product links this file; see
 * mlp_oracle.h for the list of reference lines each function follows and
 * for how parity is pinned.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).  Contraction
 * is disabled so `acc + x*w` rounds the product and the sum separately, as
 * the reference's Swift `acc += a * b` does.
 */
#include "mlp_oracle.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* half precision (Swift Float16(x) rounds to nearest even)                  */
/* ------------------------------------------------------------------------ */
uint16_t orc_f32_to_f16(float x)
{
    uint32_t u;
    memcpy(&u, &x, 4);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t ax = u & 0x7FFFFFFFu;
    if (ax > 0x7F800000u) return sign | 0x7E00u;        /* NaN */
    if (ax >= 0x477FF000u) return sign | 0x7C00u;       /* >= 65520 -> inf */
    if (ax >= 0x38800000u) {                             /* f16 normal range */
        uint32_t lsb = (ax >> 13) & 1u;
        uint32_t r = ax - 0x38000000u + 0x0FFFu + lsb;
        return sign | (uint16_t)(r >> 13);
    }
    int e = (int)(ax >> 23) - 127;                       /* f16 subnormal */
    if (e < -25) return sign;
    uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    int sh = -e - 1;                                     /* 14..24 */
    uint32_t q = m >> sh;
    uint32_t rem = m & ((1u << sh) - 1u);
    uint32_t half = 1u << (sh - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return sign | (uint16_t)q;
}

float orc_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    float v;
    if (e == 0) {
        v = ldexpf((float)m, -24);
    } else if (e == 31) {
        v = m ? NAN : INFINITY;
    } else {
        v = ldexpf((float)(m | 0x400u), (int)e - 25);
    }
    uint32_t u;
    memcpy(&u, &v, 4);
    u |= sign;
    memcpy(&v, &u, 4);
    return v;
}

/* ------------------------------------------------------------------------ */
/* E4M3 (OCP FP8 E4M3FN)                                                      */
/* ------------------------------------------------------------------------ */

/* floatToE4M3, main.swift:6-27.  Its quirks are kept on purpose: the
 * mantissa rounds half-up on magnitude using only the first dropped bit,
 * |x| < 2^-6 flushes to a signed zero (no subnormal codes), and every value
 * whose exponent reaches 15 (|x| >= 256) saturates to 0x7E (448). */
uint8_t orc_f32_to_e4m3_ref(float x)
{
    if (isnan(x)) return 0x7F;
    uint8_t sign = x < 0 ? 0x80 : 0;
    float ax = fabsf(x);
    if (ax == 0) return sign;
    if (ax >= 448.0f) return sign | 0x7E;
    uint32_t bits;
    memcpy(&bits, &ax, 4);
    int ex = (int)((bits >> 23) & 0xFFu) - 127;
    uint32_t mant = bits & 0x7FFFFFu;
    int e = ex + 7;
    if (e <= 0) return sign;
    if (e >= 15) return sign | 0x7E;
    uint32_t m3 = (mant >> 20) + ((mant >> 19) & 1u);
    if (m3 == 8) {
        m3 = 0;
        e += 1;
        if (e >= 15) return sign | 0x7E;
    }
    return (uint8_t)(sign | (uint8_t)((e << 3) | (int)m3));
}

/* OCP E4M3FN with round-to-nearest-even, subnormals, saturation to +-448.
 * Used for the seeded data mode ("N(0,1) rounded RNE to E4M3"). */
uint8_t orc_f32_to_e4m3_rne(float x)
{
    if (isnan(x)) return 0x7F;
    uint8_t sign = signbit(x) ? 0x80 : 0;
    double ax = fabs((double)x);
    if (ax >= 448.0) return sign | 0x7E;
    if (ax < 0.015625) {                        /* below 2^-6: subnormal step 2^-9 */
        double q = nearbyint(ax * 512.0);       /* exact scaling, RNE */
        return (uint8_t)(sign | (uint8_t)q);    /* q == 8 is the min normal 0x08 */
    }
    int e2;
    frexp(ax, &e2);                             /* ax = f * 2^e2, f in [0.5,1) */
    int E = e2 - 1;                             /* ax in [2^E, 2^(E+1)) */
    double q = nearbyint(ldexp(ax, 3 - E));     /* in [8, 16] */
    if (q >= 16.0) { q = 8.0; E += 1; }
    int code = ((E + 7) << 3) | ((int)q - 8);
    if (code > 0x7E) code = 0x7E;
    return (uint8_t)(sign | (uint8_t)code);
}

/* e4m3ToFloat, main.swift:30-41 (exp 0 -> m * 2^-9; 0x7F/0xFF -> NaN). */
float orc_e4m3_to_f32(uint8_t b)
{
    float s = (b & 0x80) ? -1.0f : 1.0f;
    int ex = (b >> 3) & 0x0F;
    int m = b & 0x07;
    if (ex == 0) return s * (float)m * ldexpf(1.0f, -9);
    if (ex == 15 && m == 7) return NAN;
    return s * (1.0f + (float)m / 8.0f) * ldexpf(1.0f, ex - 7);
}

/* ------------------------------------------------------------------------ */
/* E2M1 and UE8M0                                                             */
/* ------------------------------------------------------------------------ */

/* e2m1ToFloat, main.swift:44-48: 1 sign, 2 exponent, 1 mantissa, bias 1. */
float orc_e2m1_to_f32(uint8_t nibble)
{
    int e = (nibble >> 1) & 3;
    int m = nibble & 1;
    /* e == 0: subnormal m * 0.5; else (1 + m/2) * 2^(e-1) */
    float mag = (e == 0) ? 0.5f * (float)m : (1.0f + 0.5f * (float)m) * ldexpf(1.0f, e - 1);
    return (nibble & 0x8) ? -mag : mag;
}

/* e2m1Code, main.swift:50-53: a cycle over ten codes. */
uint8_t orc_e2m1_code(long i)
{
    static const uint8_t cyc[10] = {0x0, 0x1, 0x2, 0x3, 0x4, 0x5, 0x6, 0x9, 0xA, 0xC};
    return cyc[i % 10];
}

/* packE2M1, main.swift:56-67: the low nibble holds the even element. */
void orc_pack_e2m1(const uint8_t *codes, long count, uint8_t *out)
{
    for (long i = 0; i < count / 2; ++i) out[i] = 0;
    for (long i = 0; i < count; ++i) {
        uint8_t nib = codes[i] & 0xF;
        out[i / 2] |= (i % 2 == 0) ? nib : (uint8_t)(nib << 4);
    }
}

/* OCP E2M1 from f32: round to nearest, ties to the even code, on the grid
 * {0, .5, 1, 1.5, 2, 3, 4, 6}; |x| > 6 and Inf saturate to 6; NaN -> 0x7.
 * Below 2 the grid step is 0.5, in [2, 4) it is 1, from 4 on it is 2. */
uint8_t orc_f32_to_e2m1_rne(float x)
{
    if (isnan(x)) return 0x7;
    uint8_t sign = signbit(x) ? 0x8 : 0;
    double ax = fabs((double)x);
    int code;
    if (ax >= 6.0) {
        code = 7;                                 /* 6, larger values and Inf saturate */
    } else if (ax < 2.0) {
        code = (int)nearbyint(ax * 2.0);          /* 0..4 -> 0, .5, 1, 1.5, 2 */
    } else if (ax < 4.0) {
        int q = (int)nearbyint(ax);               /* 2..4 */
        code = q == 2 ? 4 : q == 3 ? 5 : 6;
    } else {
        int q = (int)nearbyint(ax / 2.0);         /* 2.. (4, 6, then saturation) */
        code = q <= 2 ? 6 : 7;
    }
    return (uint8_t)(sign | code);
}

/* OCP MX block quantisation (see the header for the exact rules). */
int orc_quantize_mx(int elem, const float *src, long rows, long cols, uint8_t *vals, uint8_t *scales)
{
    if (rows <= 0 || cols <= 0 || cols % 32 != 0 || (elem != 0 && elem != 1)) return 1;
    const int emax = elem == 0 ? 2 : 8;
    long nb = cols / 32;
    if (elem == 0) for (long i = 0; i < rows * cols / 2; ++i) vals[i] = 0;
    for (long r = 0; r < rows; ++r) {
        for (long b = 0; b < nb; ++b) {
            const float *v = src + r * cols + b * 32;
            int bad = 0;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) {
                if (!isfinite(v[i])) bad = 1;
                else if (fabsf(v[i]) > amax) amax = fabsf(v[i]);
            }
            int X;
            uint8_t code;
            if (bad) { code = 0xFF; X = 0; }
            else if (amax == 0.0f) { code = 0; X = -127; }
            else {
                int e2;
                frexpf(amax, &e2);                    /* amax in [2^(e2-1), 2^e2) */
                X = (e2 - 1) - emax;
                if (X < -127) X = -127;
                if (X > 127) X = 127;
                code = (uint8_t)(X + 127);
            }
            scales[r * nb + b] = code;
            for (int i = 0; i < 32; ++i) {
                uint8_t q = 0;
                if (!bad) {
                    float s = ldexpf(v[i], -X);       /* exact: a power-of-two scaling */
                    q = elem == 0 ? orc_f32_to_e2m1_rne(s) : orc_f32_to_e4m3_rne(s);
                }
                long idx = r * cols + b * 32 + i;
                if (elem == 0) vals[idx / 2] |= (idx % 2 == 0) ? q : (uint8_t)(q << 4);
                else vals[idx] = q;
            }
        }
    }
    return 0;
}

/* e2m1At, main.swift:69-73. */
float orc_e2m1_at(const uint8_t *packed, long index)
{
    uint8_t byte = packed[index / 2];
    uint8_t nib = (index % 2 == 0) ? (byte & 0xF) : (byte >> 4);
    return orc_e2m1_to_f32(nib);
}

/* ue8m0ToFloat, main.swift:76-78: 2^(code - 127). */
float orc_ue8m0_to_f32(uint8_t code)
{
    return ldexpf(1.0f, (int)code - 127);
}

/* ue8m0Code, main.swift:80-83: a cycle over 125..128. */
uint8_t orc_ue8m0_code(long i)
{
    return (uint8_t)(125 + (i % 4));
}

/* The E2M1 -> E4M3 widening of fp8_mlp.metal:305-309, derived here from the
 * two formats (every E2M1 value is an E4M3 value) rather than tabulated. */
uint8_t orc_e2m1_to_e4m3_byte(uint8_t nibble)
{
    float v = orc_e2m1_to_f32(nibble & 0xF);
    uint8_t b = orc_f32_to_e4m3_rne(v);
    if (nibble & 0x8) b |= 0x80;                /* -0 keeps its sign bit */
    return b;
}

/* ------------------------------------------------------------------------ */
/* operand semantics                                                          */
/* ------------------------------------------------------------------------ */

/* The dtype constraints of main.swift:370-376 and :473-476. */
int orc_check_layout(int dtype, long N, long K, long M)
{
    if (N <= 0 || K <= 0 || M <= 0) return 1;
    int fp4ok = ((N * K) % 2 == 0) && ((K * M) % 2 == 0);
    int mxok = fp4ok && (K % 32 == 0);
    if (dtype == ORC_F4F4 && !fp4ok) return 1;
    if ((dtype == ORC_MXFP4 || dtype == ORC_MX4X4) && !mxok) return 1;
    if ((dtype == ORC_MX8X4 || dtype == ORC_F8X4) && (!mxok || K % 128 != 0)) return 1;
    if (dtype < 0 || dtype >= ORC_NUM_DTYPES) return 1;
    return 0;
}

/* refActivation, main.swift:419-436. */
int orc_decode_x(int dtype, const void *X, const uint8_t *xscale,
                 long N, long K, double *out)
{
    if (orc_check_layout(dtype, N, K, 32 * 2)) return 1;
    long count = N * K;
    long kb = K / 32;
    const uint16_t *xh = (const uint16_t *)X;
    const int8_t *xi = (const int8_t *)X;
    const uint8_t *xb = (const uint8_t *)X;
    for (long i = 0; i < count; ++i) {
        long n = i / K, k = i % K;
        double v;
        switch (dtype) {
        case ORC_FP16: case ORC_INT8: case ORC_FP8: case ORC_MXFP4:
            v = orc_f16_to_f32(xh[i]); break;
        case ORC_I8I8: v = xi[i]; break;
        case ORC_F8F8: case ORC_F8X4: v = orc_e4m3_to_f32(xb[i]); break;
        case ORC_F4F4: v = orc_e2m1_at(xb, i); break;
        case ORC_MX4X4:
            v = (double)orc_e2m1_at(xb, i) * orc_ue8m0_to_f32(xscale[n * kb + k / 32]); break;
        case ORC_MX8X4:
            v = (double)orc_e4m3_to_f32(xb[i]) * orc_ue8m0_to_f32(xscale[n * kb + k / 32]); break;
        default: return 1;
        }
        out[i] = v;
    }
    return 0;
}

/* refWeight, main.swift:437-449.  The MX family stores W as [M,K] with the
 * scale plane [M, K/32]; the output is always w[k*M + m]. */
int orc_decode_w(int dtype, const void *W, const uint8_t *wscale,
                 long K, long M, double *out)
{
    if (orc_check_layout(dtype, 2, K, M)) return 1;
    long kb = K / 32;
    const uint16_t *wh = (const uint16_t *)W;
    const int8_t *wi = (const int8_t *)W;
    const uint8_t *wb = (const uint8_t *)W;
    for (long k = 0; k < K; ++k) {
        for (long m = 0; m < M; ++m) {
            long i = k * M + m;
            double v;
            switch (dtype) {
            case ORC_FP16: v = orc_f16_to_f32(wh[i]); break;
            case ORC_INT8: case ORC_I8I8: v = wi[i]; break;
            case ORC_FP8: case ORC_F8F8: v = orc_e4m3_to_f32(wb[i]); break;
            case ORC_F4F4: v = orc_e2m1_at(wb, i); break;
            case ORC_MXFP4: case ORC_MX4X4: case ORC_MX8X4: case ORC_F8X4:
                v = (double)orc_e2m1_at(wb, m * K + k) * orc_ue8m0_to_f32(wscale[m * kb + k / 32]);
                break;
            default: return 1;
            }
            out[i] = v;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* dot products                                                               */
/* ------------------------------------------------------------------------ */
void orc_dot_f64(const double *xd, const double *wd, long K, long M,
                 const long *rows, const long *cols, long count, double *out)
{
    for (long s = 0; s < count; ++s) {
        const double *xr = xd + rows[s] * K;
        long m = cols[s];
        double acc = 0.0;
        for (long k = 0; k < K; ++k) acc += xr[k] * wd[k * M + m];
        out[s] = acc;
    }
}

void orc_dot_i64(const int8_t *X, const int8_t *W, long K, long M,
                 const long *rows, const long *cols, long count, int64_t *out)
{
    for (long s = 0; s < count; ++s) {
        const int8_t *xr = X + rows[s] * K;
        long m = cols[s];
        int64_t acc = 0;
        for (long k = 0; k < K; ++k) acc += (int64_t)xr[k] * (int64_t)W[k * M + m];
        out[s] = acc;
    }
}

void orc_dot_f32_korder(const double *xd, const double *wd, long K, long M,
                        const long *rows, const long *cols, long count, float *out)
{
    for (long s = 0; s < count; ++s) {
        const double *xr = xd + rows[s] * K;
        long m = cols[s];
        float acc = 0.0f;
        for (long k = 0; k < K; ++k) {
            float p = (float)xr[k] * (float)wd[k * M + m];
            acc = acc + p;
        }
        out[s] = acc;
    }
}

/* samples(tile), main.swift:452-466. */
int orc_sample_points(long N, long M, int bm, int bn, long *rows, long *cols)
{
    long cand[6][2] = {
        {0, 0},
        {0, (bn - 1 < M - 1) ? bn - 1 : M - 1},
        {0, (bn < M - 1) ? bn : M - 1},
        {(bm - 1 < N - 1) ? bm - 1 : N - 1, 0},
        {(bm < N - 1) ? bm : N - 1, (bn < M - 1) ? bn : M - 1},
        {N - 1, M - 1},
    };
    int n = 0;
    for (int c = 0; c < 6; ++c) {
        long r = cand[c][0], q = cand[c][1];
        if (r < 0 || r >= N || q < 0 || q >= M) continue;
        int dup = 0;
        for (int j = 0; j < n; ++j) dup |= (rows[j] == r && cols[j] == q);
        if (dup) continue;
        rows[n] = r;
        cols[n] = q;
        ++n;
    }
    return n;
}

/* ------------------------------------------------------------------------ */
/* multithreaded host GEMM: the CPU baseline                                  */
/* ------------------------------------------------------------------------ */
#define ORC_RB 4     /* output rows per task (share the W stream) */
#define ORC_CB 256   /* output columns per task */

/* every processor this process may run on, whatever OMP_NUM_THREADS says
   (launchers such as torchrun set it to 1 per rank) */
int orc_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_num_procs();
#else
    return 1;
#endif
}

void orc_host_gemm_f32(const float *xf, const float *wf, long K, long M,
                       long row0, long nrows, float *Y, int nthreads)
{
    long rblocks = (nrows + ORC_RB - 1) / ORC_RB;
    long cblocks = (M + ORC_CB - 1) / ORC_CB;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_num_procs();
#pragma omp parallel for collapse(2) schedule(dynamic, 1) num_threads(nthreads)
#endif
    for (long rb = 0; rb < rblocks; ++rb) {
        for (long cb = 0; cb < cblocks; ++cb) {
            long r0 = rb * ORC_RB, c0 = cb * ORC_CB;
            int nr = (int)((nrows - r0) < ORC_RB ? (nrows - r0) : ORC_RB);
            int nc = (int)((M - c0) < ORC_CB ? (M - c0) : ORC_CB);
            float acc[ORC_RB][ORC_CB];
            for (int r = 0; r < ORC_RB; ++r)
                for (int c = 0; c < ORC_CB; ++c) acc[r][c] = 0.0f;
            for (long k = 0; k < K; ++k) {          /* K order, as the reference */
                const float *wr = wf + k * M + c0;
                for (int r = 0; r < nr; ++r) {
                    float xv = xf[(row0 + r0 + r) * K + k];
                    for (int c = 0; c < nc; ++c) acc[r][c] = acc[r][c] + xv * wr[c];
                }
            }
            for (int r = 0; r < nr; ++r)
                for (int c = 0; c < nc; ++c) Y[(r0 + r) * M + c0 + c] = acc[r][c];
        }
    }
    (void)nthreads;
}

void orc_host_gemm_i32(const int8_t *X, const int8_t *W, long K, long M,
                       long row0, long nrows, int32_t *Y, int nthreads)
{
    long rblocks = (nrows + ORC_RB - 1) / ORC_RB;
    long cblocks = (M + ORC_CB - 1) / ORC_CB;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_num_procs();
#pragma omp parallel for collapse(2) schedule(dynamic, 1) num_threads(nthreads)
#endif
    for (long rb = 0; rb < rblocks; ++rb) {
        for (long cb = 0; cb < cblocks; ++cb) {
            long r0 = rb * ORC_RB, c0 = cb * ORC_CB;
            int nr = (int)((nrows - r0) < ORC_RB ? (nrows - r0) : ORC_RB);
            int nc = (int)((M - c0) < ORC_CB ? (M - c0) : ORC_CB);
            int32_t acc[ORC_RB][ORC_CB];
            for (int r = 0; r < ORC_RB; ++r)
                for (int c = 0; c < ORC_CB; ++c) acc[r][c] = 0;
            for (long k = 0; k < K; ++k) {
                const int8_t *wr = W + k * M + c0;
                for (int r = 0; r < nr; ++r) {
                    int32_t xv = X[(row0 + r0 + r) * K + k];
                    for (int c = 0; c < nc; ++c) acc[r][c] += xv * (int32_t)wr[c];
                }
            }
            for (int r = 0; r < nr; ++r)
                for (int c = 0; c < nc; ++c) Y[(r0 + r) * M + c0 + c] = acc[r][c];
        }
    }
    (void)nthreads;
}

/* ------------------------------------------------------------------------ */
/* the reference's deterministic operands (main.swift:364-390)                */
/* ------------------------------------------------------------------------ */
/* Any output pointer may be NULL.  FP4 buffers hold count/2 bytes; the MX
 * planes hold N*(K/32) (xscale) and M*(K/32) (wscale) bytes. */
void orc_ref_operands(long N, long K, long M,
                      uint16_t *x_f16, int8_t *x_i8, uint8_t *x_e4m3, uint8_t *x_fp4,
                      uint16_t *w_f16, int8_t *w_i8, uint8_t *w_e4m3, uint8_t *w_fp4,
                      uint8_t *w_mx, uint8_t *wscale, uint8_t *xscale)
{
    long xc = N * K, wc = K * M, kb = K / 32 > 1 ? K / 32 : 1;
    for (long i = 0; i < xc; ++i) {
        float xf = (float)((i % 97) - 48) * 0.02f;
        if (x_f16) x_f16[i] = orc_f32_to_f16(xf);
        if (x_i8) x_i8[i] = (int8_t)((i % 97) - 48);
        if (x_e4m3) x_e4m3[i] = orc_f32_to_e4m3_ref(xf);
    }
    for (long i = 0; i < wc; ++i) {
        float f = (float)((i % 53) - 26) * 0.05f;
        if (w_f16) w_f16[i] = orc_f32_to_f16(f);
        if (w_i8) w_i8[i] = (int8_t)((i % 53) - 26);
        if (w_e4m3) w_e4m3[i] = orc_f32_to_e4m3_ref(f);
    }
    if (x_fp4) {
        for (long i = 0; i < xc / 2; ++i) x_fp4[i] = 0;
        for (long i = 0; i < xc; ++i)
            x_fp4[i / 2] |= (i % 2 == 0) ? orc_e2m1_code(i) : (uint8_t)(orc_e2m1_code(i) << 4);
    }
    if (w_fp4) {
        for (long i = 0; i < wc / 2; ++i) w_fp4[i] = 0;
        for (long i = 0; i < wc; ++i)
            w_fp4[i / 2] |= (i % 2 == 0) ? orc_e2m1_code(i + 3) : (uint8_t)(orc_e2m1_code(i + 3) << 4);
    }
    if (w_mx) {
        for (long i = 0; i < wc / 2; ++i) w_mx[i] = 0;
        for (long i = 0; i < wc; ++i)
            w_mx[i / 2] |= (i % 2 == 0) ? orc_e2m1_code(i + 5) : (uint8_t)(orc_e2m1_code(i + 5) << 4);
    }
    if (wscale) for (long i = 0; i < M * kb; ++i) wscale[i] = orc_ue8m0_code(i);
    if (xscale) for (long i = 0; i < N * kb; ++i) xscale[i] = orc_ue8m0_code(i + 1);
}
