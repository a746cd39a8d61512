/*
 * CPU oracle for the MXFP8 x BF16 GEMM path (D = A*B + C) and the MXFP8 codec.
 *
 * TEST INFRASTRUCTURE ONLY.  This file checks results and is not the product: only the
 * test suite, the smoke check and the benchmark's CPU-baseline leg load it.  The
 * CUDA library never calls into it and has no CPU fallback.
 *
 * It restates, in plain C, the algorithm of the reference project
 * (chcoliang/mix_precision_kernel).  Each function names the reference file:line it
 * follows.  The restatement is pinned against the reference's own host code
 * (compiled from its sources into oracle/_ref by oracle/Makefile) and against the
 * committed golden vectors in tests/golden/.
 *
 * Build: gcc -O3 -fPIC -shared -ffp-contract=off (no FMA contraction: the
 * reference's host gold performs a separately rounded multiply and add per step).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_MX_BLOCK 32              /* include/gemm_common.h:53 MXFP8_BLOCK_SIZE */
#define ORC_E4M3_MAX 448.0f          /* include/fp8_types.h:16 */
#define ORC_SCALE_FLOOR 1.1754944e-38f /* src/quantize/mxfp8_quantize.cu:131 */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------------- */
/* Scalar formats                                                             */
/* ------------------------------------------------------------------------- */

/* E4M3 code -> float, exact.  include/fp8_types.h:8-12 (E4M3 -> half -> float).
 * Layout: sign(1) exponent(4, bias 7) mantissa(3); S.1111.111 is NaN; no inf. */
float orc_e4m3_to_float(uint8_t v)
{
    int s = v >> 7, e = (v >> 3) & 15, m = v & 7;
    float mag;
    if (e == 15 && m == 7) return s ? -NAN : NAN;
    if (e == 0) mag = ldexpf((float)m, -9);             /* subnormal: m * 2^-9 */
    else        mag = ldexpf((float)(8 + m), e - 10);   /* (1 + m/8) * 2^(e-7) */
    return s ? -mag : mag;
}

/* float -> E4M3 code.  include/fp8_types.h:14-21: NaN -> 0x7F, clamp to +-448,
 * then round-to-nearest-even into E4M3 (the clamp makes saturation moot). */
uint8_t orc_float_to_e4m3(float x)
{
    if (x != x) return 0x7F;
    if (x > ORC_E4M3_MAX) x = ORC_E4M3_MAX;
    if (x < -ORC_E4M3_MAX) x = -ORC_E4M3_MAX;
    uint8_t sign = (uint8_t)((f2u(x) >> 24) & 0x80);
    float a = fabsf(x);
    if (a < 0x1p-6f) {
        /* Subnormal range: quantum 2^-9.  a*512 is exact; nearbyintf is RNE. */
        float q = nearbyintf(a * 512.0f);            /* 0..8; 8 encodes 2^-6 */
        return sign | (uint8_t)q;
    }
    int e2;
    frexpf(a, &e2);                                   /* a = f*2^e2, f in [0.5,1) */
    int E = e2 - 1;                                   /* unbiased exponent, -6..8 */
    float q = nearbyintf(ldexpf(a, 3 - E));          /* 8..16, exact scaling */
    int code = ((E + 7) << 3) + ((int)q - 8);         /* q == 16 carries */
    return sign | (uint8_t)code;
}

/* E8M0 byte -> float: bit pattern byte<<23.  include/mxfp8_utils.h:8-11.
 * Byte 0 gives 0.0 and byte 255 gives +inf (the reference's convention). */
float orc_e8m0_to_float(uint8_t b) { return u2f((uint32_t)b << 23); }

/* float -> E8M0 byte, rounding up to a power of two.  include/mxfp8_utils.h:13-22. */
uint8_t orc_float_to_e8m0(float x)
{
    if (x <= 0.0f) return 0;
    uint32_t bits = f2u(x);
    uint32_t e = (bits >> 23) & 0xFF;
    if (bits & 0x007FFFFFu) e = (e < 255) ? e + 1 : 255;
    return (uint8_t)e;
}

/* float -> bf16 bits, round-to-nearest-even; NaN -> 0x7FFF.
 * include/fp8_types.h:38-40 (__float2bfloat16). */
uint16_t orc_float_to_bf16(float x)
{
    uint32_t u = f2u(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FFF;
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

float orc_bf16_to_float(uint16_t h) { return u2f((uint32_t)h << 16); }

/* ------------------------------------------------------------------------- */
/* Worker pool helper: split [0, n) into contiguous slabs, one per thread.     */
/* ------------------------------------------------------------------------- */
typedef void (*orc_range_fn)(void* ctx, int64_t lo, int64_t hi);
typedef struct { orc_range_fn fn; void* ctx; int64_t lo, hi; } orc_job;

static void* orc_job_run(void* p)
{
    orc_job* j = (orc_job*)p;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

static void orc_parallel_for(int64_t n, int nthreads, orc_range_fn fn, void* ctx)
{
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((int64_t)nthreads > n) nthreads = (int)(n > 0 ? n : 1);
    if (nthreads == 1) { fn(ctx, 0, n); return; }
    pthread_t th[256];
    orc_job jobs[256];
    int started[256];
    for (int t = 0; t < nthreads; ++t) {
        jobs[t].fn = fn; jobs[t].ctx = ctx;
        jobs[t].lo = n * t / nthreads; jobs[t].hi = n * (t + 1) / nthreads;
        started[t] = pthread_create(&th[t], NULL, orc_job_run, &jobs[t]) == 0;
        if (!started[t]) orc_job_run(&jobs[t]);
    }
    for (int t = 0; t < nthreads; ++t)
        if (started[t]) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------- */
/* MXFP8 quantize / dequantize (blocks of 32 along the last dimension)         */
/* ------------------------------------------------------------------------- */

/* One row.  src/quantize/mxfp8_quantize.cu:120-143 (host) and :7-42 (kernel):
 * amax over the block (NaN ignored), scale = e8m0_roundup(max(amax/448, FLT_MIN)),
 * code = e4m3_rne(clamp(x * (1/scale))). */
static void orc_quantize_row(const float* in, uint8_t* data, uint8_t* scales, int64_t K)
{
    int64_t nblk = (K + ORC_MX_BLOCK - 1) / ORC_MX_BLOCK;
    for (int64_t b = 0; b < nblk; ++b) {
        int64_t k0 = b * ORC_MX_BLOCK;
        int64_t k1 = k0 + ORC_MX_BLOCK < K ? k0 + ORC_MX_BLOCK : K;
        float amax = 0.0f;
        for (int64_t k = k0; k < k1; ++k) {
            float a = fabsf(in[k]);
            if (amax < a) amax = a;                 /* std::max(amax, a): NaN ignored */
        }
        float scale_val = amax / ORC_E4M3_MAX;      /* IEEE division */
        if (scale_val < ORC_SCALE_FLOOR) scale_val = ORC_SCALE_FLOOR;
        uint8_t s = orc_float_to_e8m0(scale_val);
        float actual = orc_e8m0_to_float(s);
        scales[b] = s;
        float inv = (actual > 0.0f) ? (1.0f / actual) : 0.0f;
        for (int64_t k = k0; k < k1; ++k) data[k] = orc_float_to_e4m3(in[k] * inv);
    }
}

typedef struct { const float* in; uint8_t* data; uint8_t* scales; int64_t K, nblk; } orc_q_ctx;
static void orc_q_range(void* p, int64_t lo, int64_t hi)
{
    orc_q_ctx* c = (orc_q_ctx*)p;
    for (int64_t r = lo; r < hi; ++r)
        orc_quantize_row(c->in + r * c->K, c->data + r * c->K, c->scales + r * c->nblk, c->K);
}

void orc_mxfp8_quantize(const float* in, uint8_t* data, uint8_t* scales,
                        int64_t M, int64_t K, int nthreads)
{
    orc_q_ctx c = { in, data, scales, K, (K + ORC_MX_BLOCK - 1) / ORC_MX_BLOCK };
    orc_parallel_for(M, nthreads, orc_q_range, &c);
}

/* src/quantize/mxfp8_dequantize.cu:32-47: out = e4m3(code) * e8m0(scale). */
typedef struct { const uint8_t* data; const uint8_t* scales; float* out; int64_t K, nblk; } orc_dq_ctx;
static void orc_dq_range(void* p, int64_t lo, int64_t hi)
{
    orc_dq_ctx* c = (orc_dq_ctx*)p;
    for (int64_t r = lo; r < hi; ++r)
        for (int64_t k = 0; k < c->K; ++k) {
            float s = orc_e8m0_to_float(c->scales[r * c->nblk + k / ORC_MX_BLOCK]);
            c->out[r * c->K + k] = orc_e4m3_to_float(c->data[r * c->K + k]) * s;
        }
}

void orc_mxfp8_dequantize(const uint8_t* data, const uint8_t* scales, float* out,
                          int64_t M, int64_t K, int nthreads)
{
    orc_dq_ctx c = { data, scales, out, K, (K + ORC_MX_BLOCK - 1) / ORC_MX_BLOCK };
    orc_parallel_for(M, nthreads, orc_dq_range, &c);
}

/* ------------------------------------------------------------------------- */
/* FP32 gold GEMM: D = A*B + C                                                 */
/* ------------------------------------------------------------------------- */

/* src/reference/gemm_reference.cu:68-80 computes, per (i, j),
 *     sum = 0; for k ascending: sum = sum + A[i][k]*B[k][j]; sum = sum + C[i][j]
 * with a rounded multiply and a rounded add per step.  Looping i-k-j with one
 * float accumulator per column performs exactly the same rounded operations in
 * the same order for every (i, j), so the result is bit-identical, while reading
 * B row by row. */
static void orc_gemm_row(const float* Arow, const float* B, const float* Crow,
                         float* Drow, int64_t N, int64_t K)
{
    for (int64_t j = 0; j < N; ++j) Drow[j] = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
        const float a = Arow[k];
        const float* Bk = B + k * N;
        for (int64_t j = 0; j < N; ++j) Drow[j] = Drow[j] + a * Bk[j];
    }
    if (Crow)
        for (int64_t j = 0; j < N; ++j) Drow[j] = Drow[j] + Crow[j];
}

typedef struct {
    const float *A, *B, *C; float* D; int64_t N, K;
    const int64_t* rows;   /* NULL: all rows, D indexed by row; else D indexed by slot */
} orc_gemm_ctx;

static void orc_gemm_range(void* p, int64_t lo, int64_t hi)
{
    orc_gemm_ctx* c = (orc_gemm_ctx*)p;
    for (int64_t t = lo; t < hi; ++t) {
        int64_t i = c->rows ? c->rows[t] : t;
        orc_gemm_row(c->A + i * c->K, c->B, c->C ? c->C + i * c->N : NULL,
                     c->D + t * c->N, c->N, c->K);
    }
}

void orc_gemm_gold(const float* A, const float* B, const float* C, float* D,
                   int64_t M, int64_t N, int64_t K, int nthreads)
{
    orc_gemm_ctx c = { A, B, C, D, N, K, NULL };
    orc_parallel_for(M, nthreads, orc_gemm_range, &c);
}

/* Gold for selected rows only: D_rows[t] = row rows[t] of A*B + C.  Exact for
 * those rows, because row i of D depends only on row i of A and C and on B. */
void orc_gemm_gold_rows(const float* A, const float* B, const float* C, float* D_rows,
                        const int64_t* rows, int64_t nrows, int64_t N, int64_t K, int nthreads)
{
    orc_gemm_ctx c = { A, B, C, D_rows, N, K, rows };
    orc_parallel_for(nrows, nthreads, orc_gemm_range, &c);
}

/* ------------------------------------------------------------------------- */
/* Error metrics                                                               */
/* ------------------------------------------------------------------------- */

/* tests/test_benchmark_report.cu:123-137: rel = |res-ref| / max(|ref|, 1e-6);
 * max, mean and RMSE (accumulated here in double). */
void orc_error_stats(const float* res, const float* ref, int64_t n,
                     double* max_rel, double* avg_rel, double* rmse)
{
    double mx = 0.0, sum = 0.0, sq = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        float diff = fabsf(res[i] - ref[i]);
        float denom = fmaxf(fabsf(ref[i]), 1e-6f);
        float rel = diff / denom;
        if (rel > mx) mx = rel;
        sum += rel;
        sq += (double)diff * (double)diff;
    }
    *max_rel = mx;
    *avg_rel = n ? sum / (double)n : 0.0;
    *rmse = n ? sqrt(sq / (double)n) : 0.0;
}

/* include/gemm_common.h:39-50: max relative error over entries with |ref| > 1e-6. */
float orc_compute_relative_error(const float* res, const float* ref, int64_t n)
{
    float mx = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        if (fabsf(ref[i]) > 1e-6f) {
            float r = fabsf(res[i] - ref[i]) / fabsf(ref[i]);
            if (r > mx) mx = r;
        }
    }
    return mx;
}

/* Distance between two MXFP8 values in E4M3 steps of the coarser of the two
 * block scales: codes compared by ordinal when the scales agree, dequantized
 * values compared in units of the larger scale's quantum otherwise.  Returns a
 * histogram: hist[0] = exact, hist[1] = within one step, hist[2] = more, and
 * hist[3] = NaN mismatches. */
static int orc_e4m3_ordinal(uint8_t c)
{
    int mag = c & 0x7F;
    return (c & 0x80) ? -mag : mag;
}

static double orc_e4m3_quantum(float v, uint8_t scale)
{
    /* size of one E4M3 step at |v| for the given block scale */
    float s = orc_e8m0_to_float(scale);
    float a = fabsf(v) / s;
    int E;
    if (!(a >= 0x1p-6f)) return ldexp(1.0, -9) * s;
    frexpf(a, &E);
    return ldexp(1.0, (E - 1) - 3) * s;
}

void orc_mx_ulp_hist(const uint8_t* d1, const uint8_t* s1, const uint8_t* d2, const uint8_t* s2,
                     int64_t M, int64_t N, int64_t hist[4])
{
    int64_t nblk = (N + ORC_MX_BLOCK - 1) / ORC_MX_BLOCK;
    hist[0] = hist[1] = hist[2] = hist[3] = 0;
    for (int64_t r = 0; r < M; ++r)
        for (int64_t j = 0; j < N; ++j) {
            uint8_t a = d1[r * N + j], b = d2[r * N + j];
            uint8_t sa = s1[r * nblk + j / ORC_MX_BLOCK], sb = s2[r * nblk + j / ORC_MX_BLOCK];
            float va = orc_e4m3_to_float(a) * orc_e8m0_to_float(sa);
            float vb = orc_e4m3_to_float(b) * orc_e8m0_to_float(sb);
            if (va != va || vb != vb) { hist[(va != va && vb != vb) ? 0 : 3]++; continue; }
            if (sa == sb) {
                int d = abs(orc_e4m3_ordinal(a) - orc_e4m3_ordinal(b));
                hist[d == 0 ? 0 : (d == 1 ? 1 : 2)]++;
            } else {
                uint8_t sm = sa > sb ? sa : sb;
                double q = orc_e4m3_quantum(sa > sb ? va : vb, sm);
                double d = fabs((double)va - (double)vb);
                hist[d == 0.0 ? 0 : (d <= q * (1.0 + 1e-12) ? 1 : 2)]++;
            }
        }
}

/* Whole-range evaluation of the scalar conversion, for the exhaustive check
 * against the reference: out[i] = e4m3(bits lo + i). */
void orc_sweep_float_to_e4m3(uint64_t lo, uint64_t hi, uint8_t* out)
{
    for (uint64_t u = lo; u < hi; ++u) out[u - lo] = orc_float_to_e4m3(u2f((uint32_t)u));
}
