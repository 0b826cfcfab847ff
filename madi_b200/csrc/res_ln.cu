// res_ln.cu -- the encoder's residual + LayerNorm step beside the Q8 linear.
//
//   bias_res_ln_f16 (encoder_ops.metal:333-364):
//       X[r][i] += float(MO[r][i]) + bias[i]          (f32 residual stream, in place)
//       Y[r][i]  = half((X[r][i] - mean) * inv * gamma[i] + beta[i])
//   layer_norm_f16  (encoder_ops.metal:305-331): the same without the residual add.
//   bias_res_ln / layer_norm (encoder_ops.metal:14-120, the decoder's forms): MO
//       and Y in f32; or MO f32 and Y f16 (the decoder with f16 activations).
//   mean = sum(X[r]) / D, inv = rsqrt(sum((X[r] - mean)^2) / D + eps) (two passes;
//   the row arithmetic of ln_row.cuh).
//
// HBM-bound row kernel: one warp per row, the row held in registers (D / 128
// float4 per lane, D <= 2048) so the residual update, both reduction passes and
// the normalised output read X once.  Reductions are warp butterflies; the
// residual add keeps the reference's evaluation order ((x + mo) + bias), so X is
// bit-identical to the reference's f32 result.
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"
#include "ln_row.cuh"

namespace madi {
namespace {

constexpr int kRowsPerCta = 8;
constexpr int kMaxChunks = kLnMaxD / 128;

template <typename T> MADI_DEV float4 ld4f(const T *p);
template <> MADI_DEV float4 ld4f<float>(const float *p) { return *reinterpret_cast<const float4 *>(p); }
template <> MADI_DEV float4 ld4f<__half>(const __half *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
MADI_DEV void st4f(float *p, float a, float b, float c, float d) { *reinterpret_cast<float4 *>(p) = make_float4(a, b, c, d); }
MADI_DEV void st4f(__half *p, float a, float b, float c, float d) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(h2_as_u32(__floats2half2_rn(a, b)), h2_as_u32(__floats2half2_rn(c, d)));
}

// MT: type of MO (the projection output added to the residual); YT: type of Y.
// kN: D / 128 when fixed at compile time (D = 1280: 10), 0 for any D.  Every
// chunk's loads are predicated rather than cut off by a loop exit, so the row's
// loads are all in flight at once.  kPre (with kN fixed; used for the few rows of
// a decode step): gamma and beta, which no kernel writes, are fetched into
// registers before waiting for the previous kernel.
template <bool kRes, typename MT, typename YT, int kN, bool kPre>
__global__ void __launch_bounds__(32 * kRowsPerCta) res_ln_kernel(float *__restrict__ X, const MT *__restrict__ MO,
                                                                  const float *__restrict__ bias, YT *__restrict__ Y,
                                                                  const float *__restrict__ gamma,
                                                                  const float *__restrict__ beta, int rows, int D,
                                                                  float eps) {
    constexpr int C = kN ? kN : kMaxChunks;
    static_assert(!kPre || kN != 0, "prefetch needs a fixed width");
    constexpr int CG = kPre ? kN : 1;
    const int nch = kN ? kN : (D >> 7);
    const int row = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    pdl_trigger();
    float4 g[CG], bt[CG];
    if constexpr (kPre) {
#pragma unroll
        for (int c = 0; c < kN; ++c) {
            g[c] = *reinterpret_cast<const float4 *>(gamma + (c << 7) + (lane << 2));
            bt[c] = *reinterpret_cast<const float4 *>(beta + (c << 7) + (lane << 2));
        }
    }
    pdl_wait();                // X and MO come from the kernels before this one
    if (row >= rows) return;   // whole warps only
    float *xr = X + (size_t)row * D;
    float4 v[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
        if (c < nch) {
            const int i = (c << 7) + (lane << 2);
            float4 x = *reinterpret_cast<const float4 *>(xr + i);
            if constexpr (kRes) {
                const float4 mo = ld4f(MO + (size_t)row * D + i);
                const float4 b = *reinterpret_cast<const float4 *>(bias + i);
                x.x = (x.x + mo.x) + b.x;
                x.y = (x.y + mo.y) + b.y;
                x.z = (x.z + mo.z) + b.z;
                x.w = (x.w + mo.w) + b.w;
                *reinterpret_cast<float4 *>(xr + i) = x;
            }
            v[c] = x;
        }
    }
    float mean, inv;
    ln_row_stats<C>(v, nch, D, eps, mean, inv);
    YT *yr = Y + (size_t)row * D;
#pragma unroll
    for (int c = 0; c < C; ++c) {
        if (c < nch) {
            const int i = (c << 7) + (lane << 2);
            float4 gg, bb;
            if constexpr (kPre) {
                gg = g[c];
                bb = bt[c];
            } else {
                gg = *reinterpret_cast<const float4 *>(gamma + i);
                bb = *reinterpret_cast<const float4 *>(beta + i);
            }
            st4f(yr + i, ln_apply(v[c].x, mean, inv, gg.x, bb.x), ln_apply(v[c].y, mean, inv, gg.y, bb.y),
                 ln_apply(v[c].z, mean, inv, gg.z, bb.z), ln_apply(v[c].w, mean, inv, gg.w, bb.w));
        }
    }
}

template <typename MT, typename YT>
cudaError_t launch_ln(float *X, const MT *MO, const float *bias, YT *Y, const float *gamma, const float *beta, int rows,
                      int D, float eps, cudaStream_t st) {
    const int grid = (rows + kRowsPerCta - 1) / kRowsPerCta;
    const int blk = 32 * kRowsPerCta;
#define MADI_LN(RES, KN, PRE) \
    launch_k(res_ln_kernel<RES, MT, YT, KN, PRE>, grid, blk, 0, st, 1, X, MO, bias, Y, gamma, beta, rows, D, eps)
    if (D == 1280 && rows <= 64) return MO ? MADI_LN(true, 10, true) : MADI_LN(false, 10, true);
    if (D == 1280) return MO ? MADI_LN(true, 10, false) : MADI_LN(false, 10, false);
    return MO ? MADI_LN(true, 0, false) : MADI_LN(false, 0, false);
#undef MADI_LN
}

}  // namespace

cudaError_t launch_res_ln(float *X, const __half *MO, const float *bias, __half *Y, const float *gamma,
                          const float *beta, int rows, int D, float eps, cudaStream_t st) {
    return launch_ln<__half, __half>(X, MO, bias, Y, gamma, beta, rows, D, eps, st);
}

cudaError_t launch_res_ln_f32_y16(float *X, const float *MO, const float *bias, __half *Y, const float *gamma,
                                  const float *beta, int rows, int D, float eps, cudaStream_t st) {
    return launch_ln<float, __half>(X, MO, bias, Y, gamma, beta, rows, D, eps, st);
}

cudaError_t launch_res_ln_f32(float *X, const float *MO, const float *bias, float *Y, const float *gamma,
                              const float *beta, int rows, int D, float eps, cudaStream_t st) {
    return launch_ln<float, float>(X, MO, bias, Y, gamma, beta, rows, D, eps, st);
}

}  // namespace madi
