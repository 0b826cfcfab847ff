// res_ln.cu -- the encoder's residual + LayerNorm step beside the Q8 linear.
//
//   bias_res_ln_f16 (encoder_ops.metal:333-364):
//       X[r][i] += float(MO[r][i]) + bias[i]          (f32 residual stream, in place)
//       Y[r][i]  = half((X[r][i] - mean) * inv * gamma[i] + beta[i])
//   layer_norm_f16  (encoder_ops.metal:305-331): the same without the residual add.
//   bias_res_ln / layer_norm (encoder_ops.metal:14-120, the decoder's forms): MO
//       and Y in f32.
//   mean = sum(X[r]) / D, inv = rsqrt(sum((X[r] - mean)^2) / D + eps) (two passes).
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

namespace madi {
namespace {

constexpr int kRowsPerCta = 8;
constexpr int kMaxChunks = kLnMaxD / 128;

MADI_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

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
template <bool kRes, typename MT, typename YT>
__global__ void __launch_bounds__(32 * kRowsPerCta) res_ln_kernel(float *__restrict__ X, const MT *__restrict__ MO,
                                                                  const float *__restrict__ bias, YT *__restrict__ Y,
                                                                  const float *__restrict__ gamma,
                                                                  const float *__restrict__ beta, int rows, int D,
                                                                  float eps) {
    const int row = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;   // whole warps only
    const int nch = D >> 7;
    float *xr = X + (size_t)row * D;
    float4 v[kMaxChunks];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
        if (c >= nch) break;
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
        s += (x.x + x.y) + (x.z + x.w);
    }
    const float mean = warp_sum(s) / (float)D;
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
        if (c >= nch) break;
        const float a = v[c].x - mean, b = v[c].y - mean, cc = v[c].z - mean, d = v[c].w - mean;
        q += (a * a + b * b) + (cc * cc + d * d);
    }
    const float inv = rsqrtf(warp_sum(q) / (float)D + eps);
    YT *yr = Y + (size_t)row * D;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
        if (c >= nch) break;
        const int i = (c << 7) + (lane << 2);
        const float4 g = *reinterpret_cast<const float4 *>(gamma + i);
        const float4 bt = *reinterpret_cast<const float4 *>(beta + i);
        st4f(yr + i, (v[c].x - mean) * inv * g.x + bt.x, (v[c].y - mean) * inv * g.y + bt.y,
             (v[c].z - mean) * inv * g.z + bt.z, (v[c].w - mean) * inv * g.w + bt.w);
    }
}

}  // namespace

cudaError_t launch_res_ln(float *X, const __half *MO, const float *bias, __half *Y, const float *gamma,
                          const float *beta, int rows, int D, float eps, cudaStream_t st) {
    const int grid = (rows + kRowsPerCta - 1) / kRowsPerCta;
    if (MO)
        res_ln_kernel<true, __half, __half><<<grid, 32 * kRowsPerCta, 0, st>>>(X, MO, bias, Y, gamma, beta, rows, D, eps);
    else
        res_ln_kernel<false, __half, __half><<<grid, 32 * kRowsPerCta, 0, st>>>(X, nullptr, nullptr, Y, gamma, beta, rows,
                                                                               D, eps);
    return cudaGetLastError();
}

cudaError_t launch_res_ln_f32(float *X, const float *MO, const float *bias, float *Y, const float *gamma,
                              const float *beta, int rows, int D, float eps, cudaStream_t st) {
    const int grid = (rows + kRowsPerCta - 1) / kRowsPerCta;
    if (MO)
        res_ln_kernel<true, float, float><<<grid, 32 * kRowsPerCta, 0, st>>>(X, MO, bias, Y, gamma, beta, rows, D, eps);
    else
        res_ln_kernel<false, float, float><<<grid, 32 * kRowsPerCta, 0, st>>>(X, nullptr, nullptr, Y, gamma, beta, rows,
                                                                             D, eps);
    return cudaGetLastError();
}

}  // namespace madi
