// ln_row.cuh -- the LayerNorm of one row by one warp (encoder_ops.metal:14-67,
// :305-331): mean = sum(x) / D, inv = rsqrt(sum((x - mean)^2) / D + eps),
// y = (x - mean) * inv * gamma + beta, in f32.  Lane l holds the elements
// c * 128 + 4l .. 4l + 3 (c < nch = D / 128) as float4s.  Every operation is an
// explicitly rounded intrinsic and every sum has a fixed order, so any kernel that
// normalises rows with these helpers gives results bit-identical to the row kernel
// (res_ln.cu).
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace madi {

MADI_DEV float ln_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int C>
MADI_DEV void ln_row_stats(const float4 (&v)[C], int nch, int D, float eps, float &mean, float &inv) {
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c)
        if (c < nch) s = __fadd_rn(s, __fadd_rn(__fadd_rn(v[c].x, v[c].y), __fadd_rn(v[c].z, v[c].w)));
    mean = __fdiv_rn(ln_warp_sum(s), (float)D);
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
        if (c < nch) {
            const float a = __fsub_rn(v[c].x, mean), b = __fsub_rn(v[c].y, mean);
            const float cc = __fsub_rn(v[c].z, mean), d = __fsub_rn(v[c].w, mean);
            q = __fadd_rn(q, __fadd_rn(__fmaf_rn(a, a, __fmul_rn(b, b)), __fmaf_rn(cc, cc, __fmul_rn(d, d))));
        }
    }
    inv = rsqrtf(__fadd_rn(__fdiv_rn(ln_warp_sum(q), (float)D), eps));
}

MADI_DEV float ln_apply(float x, float mean, float inv, float g, float b) {
    return __fmaf_rn(__fmul_rn(__fsub_rn(x, mean), inv), g, b);
}

}  // namespace madi
