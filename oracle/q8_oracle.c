/*
 * q8_oracle.c -- CPU restatement of the reference's Q8_0 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path, never
 * the product: only tests/, __graft_entry__.smoke() and bench.py (its
 * cpu_baseline leg and its `--impl reference` arm) may load it.  Nothing in
 * madi_b200/ links or calls it, and the product path fails loudly when its CUDA
 * library is missing instead of falling back here.
 *
 * Reference = companyjupiter/madi, engine/metal (Zig host + Metal kernels).
 * Every function names the reference file:line it restates.
 *
 * Parity status
 *   - Quantiser (madi_orc_quantize_q8): PINNED.  tests/golden/make_golden.py runs
 *     the reference's own engine/metal/bench/quantize_q8.py (which is
 *     bit-identical to transcribe.zig quantInto by the reference's contract) on
 *     seeded F16 weights and commits its int8/f16 outputs; tests check this
 *     restatement reproduces them bit for bit.
 *   - Dequant / linear / GEMV arithmetic: parity unpinned.  The reference's
 *     kernels are Metal (Apple GPUs only) driven from Zig; neither toolchain
 *     nor GPU exists here, and the reference stores no golden tensors for this
 *     path.  These functions restate the kernels' formulas and the reference's
 *     own CPU check loops (test_q8gemm.zig:59-69, test_batchproj.zig:73-78).
 *
 * Conventions: Q8 weight = qs int8 [N][K] (K contiguous) + scales f16 [N][K/32];
 * deq(n,k) = qs[n*K+k] * scales[n*(K/32) + k/32]   (q8_gemm.metal:2-3).
 * f16 values travel as uint16_t bit patterns.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- f16 <-> f32
 * IEEE binary16, round-to-nearest-even, subnormals kept (the reference converts
 * with Zig @floatCast / Metal (half) casts, both RNE). */
float madi_orc_h2f(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff, u;
    if (e == 0) {
        if (m == 0) { u = s; }
        else {                                     /* subnormal: renormalise */
            int sh = 0;
            while (!(m & 0x400)) { m <<= 1; ++sh; }
            m &= 0x3ff;
            u = s | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        u = s | 0x7f800000u | (m << 13);
    } else {
        u = s | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f; memcpy(&f, &u, 4); return f;
}

uint16_t madi_orc_f2h(float f) {
    uint32_t u; memcpy(&u, &f, 4);
    uint32_t s = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(s | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0));
    if (a >= 0x477ff000u) return (uint16_t)(s | 0x7c00u);          /* rounds to >= 65520 -> inf */
    if (a < 0x38800000u) {                                           /* result subnormal or zero */
        if (a < 0x33000000u) return (uint16_t)s;                     /* < 2^-25: rounds to 0 */
        uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u;
        int shift = 126 - (int)e;                                    /* 14 + (113 - e) - 1 ... */
        /* value = m * 2^(e-150); target unit 2^-24 -> q = m >> (126-e) with RNE */
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) ++q;
        return (uint16_t)(s | q);
    }
    uint32_t e = (a >> 23) - 127 + 15, m = a & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13), rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) ++q;         /* carry may bump exponent: fine */
    return (uint16_t)(s | q);
}

/* ------------------------------------------------------------ quantiser (a2)
 * transcribe.zig:309-327 quantInto (and upVecQ8 :235-262, quantize_q8.py:27-40):
 * per 32-block: s = max|w| / 127 (1.0 if the block is all zero), stored as f16;
 * q = clamp(round_half_away(w * (1/s_f32)), -127, 127).  The f32 scale (not the
 * stored f16 one) drives the rounding.  q4r() is the identity for Q8. */
void madi_orc_quantize_q8(const uint16_t *w, int rows, int dim, int8_t *qs, uint16_t *scales) {
    const int nb = dim / 32;
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < nb; ++b) {
            const uint16_t *blk = w + (size_t)r * dim + (size_t)b * 32;
            float mx = 0.f;
            for (int i = 0; i < 32; ++i) { float a = fabsf(madi_orc_h2f(blk[i])); if (a > mx) mx = a; }
            float scale = mx > 0.f ? mx / 127.0f : 1.0f;
            scales[(size_t)r * nb + b] = madi_orc_f2h(scale);
            float inv = 1.0f / scale;
            for (int i = 0; i < 32; ++i) {
                float q = roundf(madi_orc_h2f(blk[i]) * inv);         /* Zig @round: half away from zero */
                if (q > 127.f) q = 127.f;
                if (q < -127.f) q = -127.f;
                qs[(size_t)r * dim + (size_t)b * 32 + i] = (int8_t)q;
            }
        }
}

/* -------------------------------------------------------------- dequant (a3)
 * q8_gemm.metal:12-27 dequant_q8_f16: out[k*N+n] = half(float(q) * float(s)),
 * transposed to [K][N].  The f32 product is exact, so this is one RNE rounding. */
static inline uint16_t deq_half(int8_t q, uint16_t s) {
    return madi_orc_f2h((float)q * madi_orc_h2f(s));
}

void madi_orc_dequant_q8_f16(const int8_t *qs, const uint16_t *scales, int N, int K, uint16_t *out) {
    const int nb = K / 32;
    for (int n = 0; n < N; ++n)
        for (int k = 0; k < K; ++k)
            out[(size_t)k * N + n] = deq_half(qs[(size_t)n * K + k], scales[(size_t)n * nb + k / 32]);
}

/* ------------------------------------------------------------------ GELU (a6)
 * m4_gemm.metal:43-57 gelu_erf == graph_helpers.metal:460-473 gelu_erf32:
 * 0.5 x (1 + erf(x/sqrt2)), erf by Abramowitz & Stegun 7.1.26 with
 * exp2(max(-z^2 log2 e, -80)).  Restated from the published formula. */
float madi_orc_gelu_erf(float xv) {
    float z = xv * 0.7071067811865476f;
    float az = fabsf(z);
    float sign = z < 0.f ? -1.f : 1.f;
    float t = 1.0f / fmaf(az, 0.3275911f, 1.0f);
    float poly = fmaf(1.061405429f, t, -1.453152027f);
    poly = fmaf(poly, t, 1.421413741f);
    poly = fmaf(poly, t, -0.284496736f);
    poly = fmaf(poly, t, 0.254829592f);
    poly = poly * t;
    float e = -az * az * 1.4426950408889634f;
    float ex = exp2f(e > -80.f ? e : -80.f);
    float erf = sign * (1.0f - poly * ex);
    return 0.5f * xv * (1.0f + erf);
}

static double gelu_d(double xv) {          /* same A&S formula, evaluated in double */
    double z = xv * 0.7071067811865476, az = fabs(z), sign = z < 0 ? -1.0 : 1.0;
    double t = 1.0 / (az * 0.3275911 + 1.0);
    double poly = ((((1.061405429 * t - 1.453152027) * t + 1.421413741) * t - 0.284496736) * t + 0.254829592) * t;
    double e = -az * az * 1.4426950408889634;
    double ex = exp2(e > -80.0 ? e : -80.0);
    return 0.5 * xv * (1.0 + sign * (1.0 - poly * ex));
}

/* Epilogue codes shared with include/madi_q8.h. */
enum { EPI_NONE = 0, EPI_BIAS = 1, EPI_BIAS_GELU = 2, EPI_BIAS_RES = 3 };

/* --------------------------------------------------------- encoder linear (a4, a5)
 * Y[m][n] = epi( sum_k X[m][k] * half(q[n][k]*s[n][k/32]) ), X f16 [M][K].
 * y_exact (f64, may be NULL): the accumulation in double over the f16-dequantised
 *   weights (q8_gemm.metal:25-26 semantics), bias added, GELU (A&S, double) or
 *   residual added -- the unrounded value the 2e-3 x RMS gate compares against.
 * y_ref (f16, may be NULL): the reference's own rounding chain -- f32 accumulate
 *   in ascending k (test_q8gemm.zig:59-69 loop order), then
 *     NONE      half(acc)                              m4_gemm_nn        m4_gemm.metal:19-41
 *     BIAS      half(float(half(acc)) + b)             m4_gemm_bias      m4_gemm.metal:60-87
 *     BIAS_GELU half(gelu(float(half(acc)) + b))       m4_gemm_bias_gelu m4_gemm.metal:89-116
 *     BIAS_RES  half(float(half(acc)) + b + float(R))  m4_gemm_nn, then the residual add of
 *                                                      bias_res_ln_f16 encoder_ops.metal:343
 * bias is f32 [N] (encoder.zig:62-72 keeps biases f32); residual f16 [M][N]. */
void madi_orc_linear_f16(const uint16_t *X, int M, int K, const int8_t *qs, const uint16_t *scales, int N,
                         const float *bias, int epi, const uint16_t *residual,
                         double *y_exact, uint16_t *y_ref) {
    const int nb = K / 32;
    float *wdq = (float *)malloc(sizeof(float) * (size_t)N * K);   /* [N][K] dequantised (half-valued) */
    for (int n = 0; n < N; ++n)
        for (int k = 0; k < K; ++k)
            wdq[(size_t)n * K + k] = madi_orc_h2f(deq_half(qs[(size_t)n * K + k], scales[(size_t)n * nb + k / 32]));
    #pragma omp parallel
    {
        float *xr = (float *)malloc(sizeof(float) * (size_t)K);
        #pragma omp for schedule(static)
        for (int m = 0; m < M; ++m) {
            for (int k = 0; k < K; ++k) xr[k] = madi_orc_h2f(X[(size_t)m * K + k]);
            for (int n = 0; n < N; ++n) {
                const float *w = wdq + (size_t)n * K;
                double accd = 0.0; float accf = 0.f;
                for (int k = 0; k < K; ++k) { accd += (double)xr[k] * (double)w[k]; accf += xr[k] * w[k]; }
                double b = (epi != EPI_NONE && bias) ? (double)bias[n] : 0.0;
                double r = (epi == EPI_BIAS_RES && residual) ? (double)madi_orc_h2f(residual[(size_t)m * N + n]) : 0.0;
                size_t o = (size_t)m * N + n;
                if (y_exact) {
                    double v = accd + b;
                    if (epi == EPI_BIAS_GELU) v = gelu_d(v);
                    y_exact[o] = v + r;
                }
                if (y_ref) {
                    float h = madi_orc_h2f(madi_orc_f2h(accf));
                    float v = h;
                    if (epi == EPI_BIAS) v = h + (float)b;
                    else if (epi == EPI_BIAS_GELU) v = madi_orc_gelu_erf(h + (float)b);
                    else if (epi == EPI_BIAS_RES) v = h + (float)b + (float)r;
                    y_ref[o] = madi_orc_f2h(v);
                }
            }
        }
        free(xr);
    }
    free(wdq);
}

/* ------------------------------------------------------- decode GEMV family (a7-a10)
 * graph_helpers.metal:390-422 gemv_q8 (and _bias :424-452, _bias_gelu :475-496,
 * _bias_res :498-519, logit_gemv_q8 :320-352): f32 throughout, no f16 rounding
 * of the weights:  out[n] = sum_p (x4[p] . q4[p]) * float(s[p/8]).
 * x f32 [M][K] (M independent token rows; M=1 is the reference's shipping case,
 * M<=8 is the batched-slot case of decoder.zig:348-403), out f32 [M][N].
 *   NONE      out = acc                (gemv_q8, logit_gemv_q8)
 *   BIAS      out = acc + b            (gemv_q8_bias)
 *   BIAS_GELU out = gelu(acc + b)      (gemv_q8_bias_gelu)
 *   BIAS_RES  out = out + acc + b      (gemv_q8_bias_res, residual in place)
 * out_exact (f64, may be NULL): double accumulation, same epilogue; for BIAS_RES
 *   it reads the residual from `out` BEFORE out_ref overwrites it.
 * out_ref (f32, may be NULL): the Metal kernel's order -- lane l (0..31) sums the
 *   char4 groups p = l, l+32, ... as ((x.x*q.x + x.y*q.y + x.z*q.z + x.w*q.w) * sc),
 *   then simd_sum (restated as an xor butterfly).  Diagnostics only. */
void madi_orc_gemv_q8(const float *x, int M, const int8_t *qs, const uint16_t *scales, int N, int K,
                      const float *bias, int epi, const float *res_in, double *out_exact, float *out_ref) {
    const int nb = K / 32, kv = K / 4;
    #pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const int8_t *q = qs + (size_t)n * K;
        const uint16_t *s = scales + (size_t)n * nb;
        for (int m = 0; m < M; ++m) {
            const float *xm = x + (size_t)m * K;
            double accd = 0.0;
            float lane[32];
            for (int l = 0; l < 32; ++l) lane[l] = 0.f;
            for (int p = 0; p < kv; ++p) {
                float sc = madi_orc_h2f(s[p >> 3]);
                const float *xv = xm + 4 * p; const int8_t *qv = q + 4 * p;
                float grp = xv[0] * (float)qv[0] + xv[1] * (float)qv[1] + xv[2] * (float)qv[2] + xv[3] * (float)qv[3];
                lane[p & 31] += grp * sc;
                for (int j = 0; j < 4; ++j) accd += (double)xv[j] * (double)qv[j] * (double)sc;
            }
            for (int off = 16; off >= 1; off >>= 1)
                for (int l = 0; l < 32; ++l) if (!(l & off)) lane[l] = lane[l] + lane[l | off];
            float accf = lane[0];
            size_t o = (size_t)m * N + n;
            float b = (epi != EPI_NONE && bias) ? bias[n] : 0.f;
            float r = (epi == EPI_BIAS_RES && res_in) ? res_in[o] : 0.f;
            if (out_exact) {
                double v = accd + (double)b;
                if (epi == EPI_BIAS_GELU) v = gelu_d(v);
                out_exact[o] = v + (double)r;
            }
            if (out_ref) {
                float v = accf + b;
                if (epi == EPI_BIAS_GELU) v = madi_orc_gelu_erf(v);
                if (epi == EPI_BIAS_RES) v = r + accf + b;
                out_ref[o] = v;
            }
        }
    }
}

/* graph_helpers.metal:527-567 gemv_q8_qkv: stacked [3D][D] weights, x f32 [M][D].
 * q = acc + qb -> q_out[m][0..D); k = acc -> kc[pos_m][.]; v = acc + vb -> vc[pos_m][.].
 * pos[m] is the KV-cache row for token row m (the reference reads one pos from
 * device memory; M rows carry one pos each).  Double accumulation. */
void madi_orc_gemv_q8_qkv(const float *x, int M, const int8_t *qs, const uint16_t *scales, int D,
                          const float *qb, const float *vb, const uint32_t *pos,
                          double *q_out, double *kc, double *vc) {
    const int nb = D / 32;
    #pragma omp parallel for schedule(static)
    for (int n = 0; n < 3 * D; ++n)
        for (int m = 0; m < M; ++m) {
            double acc = 0.0;
            for (int k = 0; k < D; ++k)
                acc += (double)x[(size_t)m * D + k] * (double)qs[(size_t)n * D + k] *
                       (double)madi_orc_h2f(scales[(size_t)n * nb + k / 32]);
            if (n < D) q_out[(size_t)m * D + n] = acc + qb[n];
            else if (n < 2 * D) kc[(size_t)pos[m] * D + (n - D)] = acc;
            else vc[(size_t)pos[m] * D + (n - 2 * D)] = acc + vb[n - 2 * D];
        }
}

/* graph_helpers.metal:64-95 (argmax_no_inc) and :785-821 (argmax_conf), restated
 * with the reference's own reduction structure: 1024 lanes, lane t scanning
 * t, t+1024, ... with a strict '>', then a halving tree (s = 512 .. 1) in which
 * slot t takes slot t+s only when strictly greater.  On ties this picks the
 * first index of the winning lane, the winning lane being the tied lane whose
 * 10-bit id is smallest when bit-reversed (NOT simply the lowest index).  When
 * conf != NULL, *conf = 1 / sum_i exp(z_i - zmax) with the same lane sums and
 * the same tree (f32, libm expf).  Returns the token. */
int madi_orc_argmax_conf(const float *logits, int V, float *conf);

int madi_orc_argmax(const float *logits, int V) {
    return madi_orc_argmax_conf(logits, V, NULL);
}

int madi_orc_argmax_conf(const float *logits, int V, float *conf) {
    float sv[1024];
    uint32_t si[1024];
    for (int t = 0; t < 1024; ++t) {
        float lm = -INFINITY;
        uint32_t li = 0;
        for (int i = t; i < V; i += 1024)
            if (logits[i] > lm) { lm = logits[i]; li = (uint32_t)i; }
        sv[t] = lm;
        si[t] = li;
    }
    for (int st = 512; st > 0; st >>= 1)
        for (int t = 0; t < st; ++t)
            if (sv[t + st] > sv[t]) { sv[t] = sv[t + st]; si[t] = si[t + st]; }
    const float zmax = sv[0];
    const uint32_t amax = si[0];
    if (conf) {
        for (int t = 0; t < 1024; ++t) {
            float ls = 0.f;
            for (int i = t; i < V; i += 1024) ls += expf(logits[i] - zmax);
            sv[t] = ls;
        }
        for (int st = 512; st > 0; st >>= 1)
            for (int t = 0; t < st; ++t) sv[t] += sv[t + st];
        *conf = 1.0f / sv[0];
    }
    return (int)amax;
}

/* graph_helpers.metal:354-383 (emb_lookup_indirect_q8 / gpu_emb_lookup_q8):
 * out[i] = float(qs[tok][i]) * float(scales[tok][i/32]) -- an exact f32 product
 * (8-bit integer times 11-bit significand).  out [dim]. */
void madi_orc_emb_q8(const int8_t *qs, const uint16_t *scales, int dim, uint32_t tok, float *out) {
    const int nb = dim / 32;
    for (int i = 0; i < dim; ++i)
        out[i] = (float)qs[(size_t)tok * dim + i] * madi_orc_h2f(scales[(size_t)tok * nb + i / 32]);
}

/* graph_helpers.metal:97-107 suppress_list: logits[ids[j]] = -3.4e38 for ids < V. */
void madi_orc_suppress(float *logits, int V, const uint32_t *ids, int n) {
    for (int j = 0; j < n; ++j)
        if (ids[j] < (uint32_t)V) logits[ids[j]] = -3.4e38f;
}

/* graph_helpers.metal:109-160 logit_filter_indirect, as one sequential pass:
 * anti-loop (three equal trailing tokens ban that token, step >= sample_begin+3),
 * windowed no-repeat-n-gram (n >= 2, last 16 tokens, a trailing (n-1)-gram seen
 * before bans the token that completed it), tokens >= 50258 banned, and space
 * (220) / EOT (50257) banned while step < sample_begin + 4.  The three bans
 * write the same constant, so their order does not change the result. */
void madi_orc_logit_filter(float *logits, int V, const uint32_t *past, uint32_t step, uint32_t sample_begin,
                           uint32_t nrng) {
    const float NEG = -3.4e38f;
    if (step >= sample_begin + 3) {
        const uint32_t t1 = past[step - 1], t2 = past[step - 2], t3 = past[step - 3];
        if (t1 == t2 && t2 == t3 && t1 < (uint32_t)V) logits[t1] = NEG;
    }
    if (nrng >= 2 && step >= sample_begin + nrng) {
        const uint32_t win = 16, suf = step - (nrng - 1);
        const uint32_t j0 = step > sample_begin + win ? step - win : sample_begin;
        for (uint32_t j = j0; j + nrng <= step; ++j) {
            int match = 1;
            for (uint32_t k = 0; k + 1 < nrng; ++k)
                if (past[j + k] != past[suf + k]) { match = 0; break; }
            if (match && past[j + nrng - 1] < (uint32_t)V) logits[past[j + nrng - 1]] = NEG;
        }
    }
    for (int t = 50258; t < V; ++t) logits[t] = NEG;
    if (step < sample_begin + 4) {
        if (220 < V) logits[220] = NEG;
        if (50257 < V) logits[50257] = NEG;
    }
}

/* ------------------------------------------------------ CPU baseline kernel
 * The reference's CPU computation for this op, timed as the CPU baseline:
 * f32 dequant-and-accumulate (test_q8gemm.zig:59-69, test_batchproj.zig:73-78)
 * with the m4_gemm epilogue, f16 out.  Rows of X are spread over `nthreads`
 * OpenMP threads; the inner loop is plain f32 (vectorised by the compiler).
 * Y f16 [M][N].  Returns 0. */
int madi_orc_linear_f32_baseline(const uint16_t *X, int M, int K, const int8_t *qs, const uint16_t *scales,
                                 int N, const float *bias, int epi, const uint16_t *residual,
                                 uint16_t *Y, int nthreads) {
    const int nb = K / 32;
    float *wdq = (float *)malloc(sizeof(float) * (size_t)N * K);
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int n = 0; n < N; ++n)
        for (int k = 0; k < K; ++k)
            wdq[(size_t)n * K + k] = (float)qs[(size_t)n * K + k] * madi_orc_h2f(scales[(size_t)n * nb + k / 32]);
    #pragma omp parallel num_threads(nthreads)
    {
        float *xr = (float *)malloc(sizeof(float) * (size_t)K);
        #pragma omp for schedule(static)
        for (int m = 0; m < M; ++m) {
            for (int k = 0; k < K; ++k) xr[k] = madi_orc_h2f(X[(size_t)m * K + k]);
            for (int n = 0; n < N; ++n) {
                const float *w = wdq + (size_t)n * K;
                float acc = 0.f;
                #pragma omp simd reduction(+:acc)
                for (int k = 0; k < K; ++k) acc += xr[k] * w[k];
                float v = acc;
                if (epi != EPI_NONE && bias) v += bias[n];
                if (epi == EPI_BIAS_GELU) v = madi_orc_gelu_erf(v);
                if (epi == EPI_BIAS_RES && residual) v += madi_orc_h2f(residual[(size_t)m * N + n]);
                Y[(size_t)m * N + n] = madi_orc_f2h(v);
            }
        }
        free(xr);
    }
    free(wdq);
    return 0;
}

/* bias_res_ln_f16 (encoder_ops.metal:333-364) / layer_norm_f16 (:305-331).
 * x[r][i] += float(mo[r][i]) + bias[i] in f32 in the reference's order
 * ((x + mo) + bias: encoder_ops.metal:347), then the LayerNorm of the updated
 * row -- mean, two-pass variance, rsqrt(var + eps), * gamma + beta -- in double:
 * y_exact is the unrounded value the f16 output is checked against.  mo == NULL
 * restates layer_norm_f16 (x unchanged). */
void madi_orc_bias_res_ln(float *x, const uint16_t *mo, const float *bias, const float *gamma, const float *beta,
                          int rows, int d, float eps, double *y_exact) {
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        float *xr = x + (size_t)r * d;
        if (mo) {
            const uint16_t *mr = mo + (size_t)r * d;
            for (int i = 0; i < d; ++i) xr[i] = (xr[i] + madi_orc_h2f(mr[i])) + bias[i];
        }
        double mean = 0.0;
        for (int i = 0; i < d; ++i) mean += (double)xr[i];
        mean /= d;
        double var = 0.0;
        for (int i = 0; i < d; ++i) { const double t = (double)xr[i] - mean; var += t * t; }
        var /= d;
        const double inv = 1.0 / sqrt(var + (double)eps);
        double *yr = y_exact + (size_t)r * d;
        for (int i = 0; i < d; ++i) yr[i] = ((double)xr[i] - mean) * inv * (double)gamma[i] + (double)beta[i];
    }
}

int madi_orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
