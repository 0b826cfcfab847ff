// q8_misc.cu -- the two byte/integer kernels beside the linear:
//   dequant_q8_f16  (q8_gemm.metal:12-27)   Q8 [N][K] -> f16 [K][N], transposed
//   quantize        (transcribe.zig:309-327) f16 [rows][dim] -> Q8 (int8 + f16 scales)
// Both are HBM-bound.  This file is compiled without fast-math so the
// quantiser's divisions and rounding are IEEE-exact (bit parity with the
// reference's f32 arithmetic).
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"

namespace madi {
namespace {

// 64 (n) x 64 (k) tile per 256-thread CTA.  Reads 16 int8 per thread along k
// (coalesced rows of the Q8 matrix), transposes through shared memory, writes
// 16-byte f16 runs along n (coalesced rows of the [K][N] output).
constexpr int TN = 64, TK = 64;

__global__ void __launch_bounds__(256) dequant_f16_kernel(const int8_t *__restrict__ qs,
                                                          const __half *__restrict__ scales, int N, int K,
                                                          __half *__restrict__ out) {
    __shared__ __half tile[TK][TN + 8];
    const int n0 = blockIdx.x * TN, k0 = blockIdx.y * TK;
    const int nkb = K / 32;
    {
        const int row = threadIdx.x >> 2, c = threadIdx.x & 3;   // 64 rows x 4 chunks of 16
        const int n = n0 + row, k = k0 + c * 16;
        if (n < N && k < K) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(qs + (size_t)n * K + k));
            const __half2 sc = __half2half2(scales[(size_t)n * nkb + (k >> 5)]);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                __half2 lo, hi;
                q8_to_half2x2(w[i], lo, hi);
                lo = __hmul2(lo, sc);   // half(q * s): one RNE rounding, as half(float(q)*float(s))
                hi = __hmul2(hi, sc);
                tile[c * 16 + 4 * i + 0][row] = __low2half(lo);
                tile[c * 16 + 4 * i + 1][row] = __high2half(lo);
                tile[c * 16 + 4 * i + 2][row] = __low2half(hi);
                tile[c * 16 + 4 * i + 3][row] = __high2half(hi);
            }
        }
    }
    __syncthreads();
    // 64 k-rows x 8 runs of 8 halves
    for (int i = threadIdx.x; i < TK * (TN / 8); i += 256) {
        const int kr = i >> 3, run = i & 7;
        const int k = k0 + kr, n = n0 + run * 8;
        if (k >= K) continue;
        __half *dst = out + (size_t)k * N + n;
        if (n + 8 <= N && (N & 7) == 0) {
            uint4 v;
            v.x = *reinterpret_cast<const uint32_t *>(&tile[kr][run * 8 + 0]);
            v.y = *reinterpret_cast<const uint32_t *>(&tile[kr][run * 8 + 2]);
            v.z = *reinterpret_cast<const uint32_t *>(&tile[kr][run * 8 + 4]);
            v.w = *reinterpret_cast<const uint32_t *>(&tile[kr][run * 8 + 6]);
            *reinterpret_cast<uint4 *>(dst) = v;
        } else {
            for (int j = 0; j < 8 && n + j < N; ++j) dst[j] = tile[kr][run * 8 + j];
        }
    }
}

// One warp per 32-element block: lane i owns element i.
//   s = max|w| / 127 (1.0 for an all-zero block), stored f16;
//   q = clamp(round_half_away(w * (1/s)), +-127) with the f32 s.
__global__ void __launch_bounds__(256) quantize_kernel(const __half *__restrict__ w, long long nblocks,
                                                       int8_t *__restrict__ qs, __half *__restrict__ scales) {
    const long long blk = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (blk >= nblocks) return;
    const int lane = threadIdx.x & 31;
    const float v = __half2float(w[blk * 32 + lane]);
    float mx = fabsf(v);
#pragma unroll
    for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    float q = roundf(__fmul_rn(v, inv));
    q = fminf(fmaxf(q, -127.0f), 127.0f);
    qs[blk * 32 + lane] = (int8_t)(int)q;
    if (lane == 0) scales[blk] = __float2half_rn(scale);
}

}  // namespace

cudaError_t launch_dequant_f16(const int8_t *qs, const __half *scales, int N, int K, __half *out, cudaStream_t st) {
    dim3 grid((N + TN - 1) / TN, (K + TK - 1) / TK);
    dequant_f16_kernel<<<grid, 256, 0, st>>>(qs, scales, N, K, out);
    return cudaGetLastError();
}

cudaError_t launch_quantize_f16(const __half *w, int rows, int dim, int8_t *qs, __half *scales, cudaStream_t st) {
    const long long nblocks = (long long)rows * (dim / 32);
    const long long grid = (nblocks + 7) / 8;
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    quantize_kernel<<<(unsigned)grid, 256, 0, st>>>(w, nblocks, qs, scales);
    return cudaGetLastError();
}

}  // namespace madi
