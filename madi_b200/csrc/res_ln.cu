// res_ln.cu -- the encoder's residual + LayerNorm step beside the Q8 linear.
//
//   bias_res_ln_f16 (encoder_ops.metal:333-364):
//       X[r][i] += float(MO[r][i]) + bias[i]          (f32 residual stream, in place)
//       Y[r][i]  = half((X[r][i] - mean) * inv * gamma[i] + beta[i])
//   layer_norm_f16  (encoder_ops.metal:305-331): the same without the residual add.
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

template <bool kRes>
__global__ void __launch_bounds__(32 * kRowsPerCta) res_ln_kernel(float *__restrict__ X, const __half *__restrict__ MO,
                                                                  const float *__restrict__ bias, __half *__restrict__ Y,
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
            const uint2 mo = *reinterpret_cast<const uint2 *>(MO + (size_t)row * D + i);
            const float4 b = *reinterpret_cast<const float4 *>(bias + i);
            const __half2 m01 = *reinterpret_cast<const __half2 *>(&mo.x);
            const __half2 m23 = *reinterpret_cast<const __half2 *>(&mo.y);
            x.x = (x.x + __low2float(m01)) + b.x;
            x.y = (x.y + __high2float(m01)) + b.y;
            x.z = (x.z + __low2float(m23)) + b.z;
            x.w = (x.w + __high2float(m23)) + b.w;
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
    __half *yr = Y + (size_t)row * D;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
        if (c >= nch) break;
        const int i = (c << 7) + (lane << 2);
        const float4 g = *reinterpret_cast<const float4 *>(gamma + i);
        const float4 bt = *reinterpret_cast<const float4 *>(beta + i);
        const __half2 y01 = __floats2half2_rn((v[c].x - mean) * inv * g.x + bt.x, (v[c].y - mean) * inv * g.y + bt.y);
        const __half2 y23 = __floats2half2_rn((v[c].z - mean) * inv * g.z + bt.z, (v[c].w - mean) * inv * g.w + bt.w);
        *reinterpret_cast<uint2 *>(yr + i) = make_uint2(h2_as_u32(y01), h2_as_u32(y23));
    }
}

}  // namespace

cudaError_t launch_res_ln(float *X, const __half *MO, const float *bias, __half *Y, const float *gamma,
                          const float *beta, int rows, int D, float eps, cudaStream_t st) {
    const int grid = (rows + kRowsPerCta - 1) / kRowsPerCta;
    if (MO)
        res_ln_kernel<true><<<grid, 32 * kRowsPerCta, 0, st>>>(X, MO, bias, Y, gamma, beta, rows, D, eps);
    else
        res_ln_kernel<false><<<grid, 32 * kRowsPerCta, 0, st>>>(X, nullptr, nullptr, Y, gamma, beta, rows, D, eps);
    return cudaGetLastError();
}

}  // namespace madi
