/*
 * cpu_baseline.c -- the reference's CPU computation of the Q8 linear, timed as
 * the CPU baseline beside the GPU numbers.
 *
 * TEST / MEASUREMENT INFRASTRUCTURE ONLY, like q8_oracle.c: only bench.py's
 * cpu_baseline leg and its `--impl reference` arm load it.  Nothing in madi_b200/
 * links or calls it.
 *
 * The reference's own CPU loop for this op is the f32 dequant-and-accumulate of
 * engine/metal/test_q8gemm.zig:59-69 (same loop: test_batchproj.zig:73-78):
 *     acc = 0; for k: acc += x[m][k] * (float(q[n][k]) * float(s[n][k/32]))
 * with the m4_gemm epilogue (m4_gemm.metal:60-116: + bias, A&S GELU, + residual)
 * and an f16 result.  Three forms, all with that arithmetic:
 *   madi_cpu_linear_faithful  the loop exactly as written: one thread, k ascending,
 *                             scalar f32, dequant inline;
 *   madi_cpu_linear_tiled     the same sums on all host cores: weights dequantised
 *                             to f32 ONCE per run (madi_cpu_dequant_f32; a decode
 *                             or encoder run amortises it over every token), then a
 *                             register-tiled kernel (4 rows x 4 outputs per tile
 *                             with AVX-512, 3 x 3 with AVX2; vectorised along k,
 *                             OpenMP over output blocks);
 *   madi_cpu_gemv_q8          the decode projection at M <= 16 token rows
 *                             (graph_helpers.metal:390-519 semantics, f32 out):
 *                             memory-bound, so int8 weights are read as they are
 *                             and dequantised in registers, every weight row
 *                             serving all M rows.
 * Built per host with -O3 -march=native -fopenmp -ffp-contract=fast (oracle/Makefile,
 * target `native`), so the vector width and FMA are the box's own; the faithful
 * loop alone keeps separate multiplies and adds.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

float madi_orc_h2f(uint16_t h);
uint16_t madi_orc_f2h(float f);
float madi_orc_gelu_erf(float x);

enum { EPI_NONE = 0, EPI_BIAS = 1, EPI_BIAS_GELU = 2, EPI_BIAS_RES = 3 };

#if defined(__AVX512F__)
#define VW 16
#define TR 4           /* token rows per register tile */
#define TC 4           /* outputs per register tile */
#else
#define VW 8
#define TR 3
#define TC 3
#endif
typedef float vf __attribute__((vector_size(VW * 4)));

/* f16 -> f32 through the compiler's _Float16 (F16C on x86-64): exact */
static inline float h2f(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

static inline float hsum(vf v) {
    float s = 0.f;
    for (int i = 0; i < VW; ++i) s += v[i];
    return s;
}

static inline vf vload(const float *p) {
    vf v;
    memcpy(&v, p, sizeof v);
    return v;
}

static inline uint16_t epilogue(float v, int n, const float *bias, int epi, const uint16_t *res_row) {
    if (epi != EPI_NONE && bias) v += bias[n];
    if (epi == EPI_BIAS_GELU) v = madi_orc_gelu_erf(v);
    if (epi == EPI_BIAS_RES && res_row) v += madi_orc_h2f(res_row[n]);
    return madi_orc_f2h(v);
}

int madi_cpu_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* test_q8gemm.zig:59-69 as written: one thread, scalar, k ascending, no fused
 * multiply-add (Zig's strict float mode). */
__attribute__((optimize("fp-contract=off")))
void madi_cpu_linear_faithful(const uint16_t *X, int M, int K, const int8_t *qs, const uint16_t *scales, int N,
                              const float *bias, int epi, const uint16_t *residual, uint16_t *Y) {
    const int nb = K / 32;
    float *xr = (float *)malloc(sizeof(float) * (size_t)K);
    for (int m = 0; m < M; ++m) {
        for (int k = 0; k < K; ++k) xr[k] = madi_orc_h2f(X[(size_t)m * K + k]);
        for (int n = 0; n < N; ++n) {
            const int8_t *q = qs + (size_t)n * K;
            const uint16_t *s = scales + (size_t)n * nb;
            float acc = 0.f;
            for (int k = 0; k < K; ++k) acc += xr[k] * ((float)q[k] * madi_orc_h2f(s[k / 32]));
            Y[(size_t)m * N + n] = epilogue(acc, n, bias, epi, residual ? residual + (size_t)m * N : NULL);
        }
    }
    free(xr);
}

/* wdq[n][k] = float(q) * float(s): the dequant the reference's loop does inline,
 * hoisted out of the token loop (done once per run). */
void madi_cpu_dequant_f32(const int8_t *qs, const uint16_t *scales, int N, int K, float *wdq, int nthreads) {
    const int nb = K / 32;
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int n = 0; n < N; ++n)
        for (int k = 0; k < K; ++k)
            wdq[(size_t)n * K + k] = (float)qs[(size_t)n * K + k] * h2f(scales[(size_t)n * nb + k / 32]);
}

/* All host cores.  X f16 [M][K] is widened to f32 once per call; output blocks of
 * 64 weight rows (their f32 rows stay in the core's L2) x all token rows are
 * spread over the threads; inside a block, TR x TC register tiles run along k in
 * vectors of VW.  K % VW == 0. */
void madi_cpu_linear_tiled(const uint16_t *X, int M, int K, const float *wdq, int N, const float *bias, int epi,
                           const uint16_t *residual, uint16_t *Y, int nthreads) {
    float *xf = (float *)malloc(sizeof(float) * (size_t)M * K);
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (long long i = 0; i < (long long)M * K; ++i) xf[i] = h2f(X[i]);
    const int NB = 64;
    const int nblk = (N + NB - 1) / NB;
    #pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
    for (int b = 0; b < nblk; ++b) {
        const int n0 = b * NB, n1 = n0 + NB < N ? n0 + NB : N;
        for (int m0 = 0; m0 < M; m0 += TR) {
            const int mr = M - m0 < TR ? M - m0 : TR;
            for (int nn = n0; nn < n1; nn += TC) {
                const int nc = n1 - nn < TC ? n1 - nn : TC;
                vf acc[TR][TC];
                memset(acc, 0, sizeof acc);
                const float *xrow[TR], *wrow[TC];
                for (int r = 0; r < TR; ++r) xrow[r] = xf + (size_t)(m0 + (r < mr ? r : 0)) * K;
                for (int c = 0; c < TC; ++c) wrow[c] = wdq + (size_t)(nn + (c < nc ? c : 0)) * K;
                for (int k = 0; k < K; k += VW) {
                    vf xv[TR], wv[TC];
                    for (int r = 0; r < TR; ++r) xv[r] = vload(xrow[r] + k);
                    for (int c = 0; c < TC; ++c) wv[c] = vload(wrow[c] + k);
                    for (int r = 0; r < TR; ++r)
                        for (int c = 0; c < TC; ++c) acc[r][c] += xv[r] * wv[c];
                }
                for (int r = 0; r < mr; ++r) {
                    const int m = m0 + r;
                    for (int c = 0; c < nc; ++c)
                        Y[(size_t)m * N + nn + c] = epilogue(hsum(acc[r][c]), nn + c, bias, epi,
                                                             residual ? residual + (size_t)m * N : NULL);
                }
            }
        }
    }
    free(xf);
}

/* Decode projection, f32 in / f32 out: y[m][n] = epi(sum_k x[m][k] * q[n][k] * s[n][k/32]),
 * epi as the gemv_q8 family (bias; bias + GELU; y = y + acc + bias for BIAS_RES).
 * M <= 16, K % 32 == 0, K <= 8192.  Each weight row is read once and serves all M rows; the
 * row count is a compile-time constant in the loop body (GEMV_ROWS) so the M
 * accumulators stay in registers. */
typedef signed char vc8 __attribute__((vector_size(VW)));
typedef int vi __attribute__((vector_size(VW * 4)));

static inline void gemv_finish(float v, int m, int n, int N, const float *bias, int epi, float *y) {
    if (epi != EPI_NONE && bias) v += bias[n];
    if (epi == EPI_BIAS_GELU) v = madi_orc_gelu_erf(v);
    if (epi == EPI_BIAS_RES) v += y[(size_t)m * N + n];
    y[(size_t)m * N + n] = v;
}

#define GEMV_ROWS(MR)                                                                              \
    static void gemv_rows_##MR(const float *x, const int8_t *qs, const uint16_t *scales, int N, int K, \
                               const float *bias, int epi, float *y, int nthreads) {               \
        const int nb = K / 32;                                                                     \
        _Pragma("omp parallel for num_threads(nthreads) schedule(static)")                         \
        for (int n = 0; n < N; ++n) {                                                              \
            vf acc[MR];                                                                            \
            const int8_t *q = qs + (size_t)n * K;                                                  \
            float sf[256];                                                                         \
            for (int b = 0; b < nb; ++b) sf[b] = h2f(scales[(size_t)n * nb + b]);                  \
            for (int m = 0; m < MR; ++m) acc[m] = (vf){0};                                         \
            for (int b = 0; b < nb; ++b) {                                                         \
                const float s = sf[b];                                                             \
                for (int j = 0; j < 32; j += VW) {                                                 \
                    vc8 qv;                                                                        \
                    memcpy(&qv, q + b * 32 + j, sizeof qv);                                        \
                    const vf w = __builtin_convertvector(__builtin_convertvector(qv, vi), vf) * s;                              \
                    for (int m = 0; m < MR; ++m) acc[m] += vload(x + (size_t)m * K + b * 32 + j) * w; \
                }                                                                                  \
            }                                                                                      \
            for (int m = 0; m < MR; ++m) gemv_finish(hsum(acc[m]), m, n, N, bias, epi, y);         \
        }                                                                                          \
    }
GEMV_ROWS(1)
GEMV_ROWS(2)
GEMV_ROWS(4)
GEMV_ROWS(8)
GEMV_ROWS(16)

void madi_cpu_gemv_q8(const float *x, int M, const int8_t *qs, const uint16_t *scales, int N, int K,
                      const float *bias, int epi, float *y, int nthreads) {
    /* M rows in groups the unrolled bodies take: 16, 8, 4, 2, 1 */
    int m0 = 0;
    while (m0 < M) {
        const int r = M - m0;
        const float *xm = x + (size_t)m0 * K;
        float *ym = y + (size_t)m0 * N;
        if (r >= 16) { gemv_rows_16(xm, qs, scales, N, K, bias, epi, ym, nthreads); m0 += 16; }
        else if (r >= 8) { gemv_rows_8(xm, qs, scales, N, K, bias, epi, ym, nthreads); m0 += 8; }
        else if (r >= 4) { gemv_rows_4(xm, qs, scales, N, K, bias, epi, ym, nthreads); m0 += 4; }
        else if (r >= 2) { gemv_rows_2(xm, qs, scales, N, K, bias, epi, ym, nthreads); m0 += 2; }
        else { gemv_rows_1(xm, qs, scales, N, K, bias, epi, ym, nthreads); m0 += 1; }
    }
}
