// q8_gemv_rows.cu -- variant (b) for K <= 1280 (every decoder projection but fc2,
// and the vocab head): the decode Q8_0 GEMV / skinny GEMM with one WARP per unit of
// 8 weight rows over the whole of K, so no partial sums cross warps and no block-wide
// barrier runs per unit.
//
// Arithmetic (graph_helpers.metal:320-567, f32 semantics), as q8_gemv_tile.cu: int8
// weights become f16 exactly, each 32-block's products meet in one f32 accumulator
// (mma.sync m16n8k16, f32), the block's f16 scale is applied in f32, the blocks are
// summed in k order.  Roles in the MMA are swapped against q8_gemv_tile.cu: A (16 x
// 16) holds the activations -- token rows 0..7, and rows 8..15 for tokens 8..15 or,
// for f32 x, the low halves of the same 8 tokens (x = hi + lo, both f16, ~22 mantissa
// bits) -- and B (16 x 8) the 8 weight rows of the unit, so one B fragment (4 int8 per
// lane, one conversion) feeds one MMA and every lane's accumulators belong to its own
// two weight rows.
//
// Data movement:
//   * a unit's weights arrive by TMA as K/256 boxes of [8 rows][2][128 B] under the
//     128-byte swizzle (the weights viewed as [N][K/128][128]), plus one [8][K/32] box
//     of scales; rows past N arrive zero-filled.  Lane (g, t) reads 8 bytes of row g
//     per 32-block (k = 8t .. 8t+7 of the block: the two k16 steps); inside a box its
//     8 byte offsets are constants, and the swizzle puts the four rows a half-warp
//     reads in different bank groups (conflict-free);
//   * x is staged once per CTA as [32-block][16 rows][4] chunks of 8 halves, so lane
//     (g, t) takes its A fragments for both k16 steps with one 16-byte load;
//   * a ring of 16 stages, two per consumer warp: the CTA's units go round robin to
//     its 8 consumer warps (unit j -> warp j mod 8, stage j mod 16), each CTA owning a
//     contiguous range of units (counts differ by at most one).  One producer warp
//     keeps every stage in flight; it runs ahead of griddepcontrol.wait (weights do
//     not depend on the previous kernel).
// One CTA per SM (about 200 KB of shared memory); grid = min(SMs, units).  Every
// wait is bounded.  Results do not depend on N, M or the grid: each output is its
// row's own k-ordered sum.
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>

#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace madi {
namespace {

constexpr int kRW = 8;                          // consumer warps per CTA
constexpr int kRThreads = 32 * (kRW + 1);
constexpr int kRRows = 8;                       // weight rows per unit (the MMA's n)
constexpr int kRStages = 2 * kRW;               // two stages per consumer warp
constexpr int kRMaxK = 1280;
constexpr int kRBox = kRRows * 256;             // one [8][2][128 B] weight box

// x staging modes
constexpr int kX16 = 0;      // f16 x (or f32 rounded to f16), tokens 0..7
constexpr int kX16W = 1;     // f16 x (or f32 rounded), tokens 0..15
constexpr int kX32 = 2;      // f32 x split hi + lo, tokens 0..7

struct __align__(8) RowBars {
    uint64_t full[kRStages];
    uint64_t empty[kRStages];
    int abort;
};

__host__ __device__ constexpr size_t rstage_bytes(int K) {
    return ((size_t)kRRows * K + (size_t)kRRows * (K / 32) * 2 + 1023) & ~size_t(1023);
}
__host__ __device__ constexpr int rx_rows(int mode) { return mode == kX16 ? 8 : 16; }
__host__ __device__ constexpr size_t rx_bytes(int K, int mode) { return (size_t)(K / 32) * rx_rows(mode) * 64; }
size_t rows_smem(int K, int mode) { return 1024 + kRStages * rstage_bytes(K) + rx_bytes(K, mode) + sizeof(RowBars); }

MADI_DEV void mma16816z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    const float z = 0.f;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}
MADI_DEV void mma16816a(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T> MADI_DEV float r_to_f32(T v);
template <> MADI_DEV float r_to_f32<float>(float v) { return v; }
template <> MADI_DEV float r_to_f32<__half>(__half v) { return __half2float(v); }
template <typename T> MADI_DEV T r_from_f32(float v);
template <> MADI_DEV float r_from_f32<float>(float v) { return v; }
template <> MADI_DEV __half r_from_f32<__half>(float v) { return __float2half_rn(v); }

// One output: y[tok][row] (or the QKV routing of gemv_q8_qkv, graph_helpers.metal:527-567).
template <typename YT, int EPI, bool kQKV>
MADI_DEV void store_one(const GemvArgs &p, int row, int tok, float y) {
    if (row >= p.N || tok >= p.M) return;
    if constexpr (kQKV) {
        const int D = p.D;
        if (row < D) {
            reinterpret_cast<float *>(p.y)[(size_t)tok * D + row] = y + p.qb[row];
        } else {
            const size_t base = (size_t)tok * p.cache_stride + (size_t)p.pos[tok] * D;
            if (row < 2 * D) p.kc[base + (row - D)] = y;
            else p.vc[base + (row - 2 * D)] = y + p.vb[row - 2 * D];
        }
    } else {
        float b = 0.f;
        if constexpr (EPI != kEpiNone)
            b = p.bias_f16 ? __half2float(reinterpret_cast<const __half *>(p.bias)[row])
                           : reinterpret_cast<const float *>(p.bias)[row];
        const size_t o = (size_t)tok * p.N + row;
        if constexpr (EPI == kEpiBias) y = y + b;
        if constexpr (EPI == kEpiBiasGelu) y = gelu_erf(y + b);
        if constexpr (EPI == kEpiBiasRes) y = r_to_f32(reinterpret_cast<const YT *>(p.residual)[o]) + y + b;
        reinterpret_cast<YT *>(p.y)[o] = r_from_f32<YT>(y);
    }
}

// x -> shared memory: chunk (b, r, t) = 8 halves for k = 32b + 8t .. +7 of row r.
// Rows past M (and, for kX32, rows 8..15 = the low halves of tokens 0..7) as the
// mode says.  Read on the coherent L2 path: under programmatic dependent launch x
// may come from a kernel that overlaps this one.
template <typename XT, int kMode>
MADI_DEV void stage_x_rows(const GemvArgs &p, uint4 *xs, int tid, int nthr) {
    constexpr int R = rx_rows(kMode);
    const int nkb = p.K >> 5, M = p.M, K = p.K;
    const int total = nkb * R * 4;
    for (int c = tid; c < total; c += nthr) {
        const int t = c & 3, r = (c >> 2) % R, b = (c >> 2) / R;
        const int tok = kMode == kX32 ? (r & 7) : r;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (tok < M) {
            const size_t k = (size_t)b * 32 + 8 * t;
            if constexpr (sizeof(XT) == 2) {
                v = __ldcg(reinterpret_cast<const uint4 *>(reinterpret_cast<const __half *>(p.x) + (size_t)tok * K + k));
            } else {
                const float4 *src = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p.x) +
                                                                     (size_t)tok * K + k);
                const float4 f0 = __ldcg(src), f1 = __ldcg(src + 1);
                __half2 h[4] = {__floats2half2_rn(f0.x, f0.y), __floats2half2_rn(f0.z, f0.w),
                                __floats2half2_rn(f1.x, f1.y), __floats2half2_rn(f1.z, f1.w)};
                if (kMode == kX32 && r >= 8) {          // low halves: x - f16(x), rounded to f16
                    h[0] = __floats2half2_rn(f0.x - __low2float(h[0]), f0.y - __high2float(h[0]));
                    h[1] = __floats2half2_rn(f0.z - __low2float(h[1]), f0.w - __high2float(h[1]));
                    h[2] = __floats2half2_rn(f1.x - __low2float(h[2]), f1.y - __high2float(h[2]));
                    h[3] = __floats2half2_rn(f1.z - __low2float(h[3]), f1.w - __high2float(h[3]));
                }
                v = make_uint4(h2_as_u32(h[0]), h2_as_u32(h[1]), h2_as_u32(h[2]), h2_as_u32(h[3]));
            }
        }
        xs[c] = v;
    }
}

template <typename XT, typename YT, int EPI, bool kQKV, int kMode>
__global__ void __launch_bounds__(kRThreads, 1)
    q8_gemv_rows_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tms,
                        const GemvArgs p, int *dev_err) {
    constexpr int R = rx_rows(kMode);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int K = p.K, nkb = K >> 5, nbox = K >> 8;
    const size_t sb = rstage_bytes(K);
    uint8_t *ring = smem;
    uint4 *xs = reinterpret_cast<uint4 *>(smem + (size_t)kRStages * sb);
    RowBars *bars = reinterpret_cast<RowBars *>(reinterpret_cast<uint8_t *>(xs) + rx_bytes(K, kMode));
    volatile int *abort_flag = &bars->abort;

    // this CTA's contiguous range of units
    const int units = (p.N + kRRows - 1) / kRRows;
    const int base = units / (int)gridDim.x, rem = units % (int)gridDim.x;
    const int cta = (int)blockIdx.x;
    const int u0 = cta * base + (cta < rem ? cta : rem);
    const int nu = base + (cta < rem ? 1 : 0);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        bars->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------ producer
        if (lane == 0) {
            tma_prefetch_desc(&tmq);
            tma_prefetch_desc(&tms);
            const uint32_t tx = (uint32_t)nbox * kRBox + (uint32_t)kRRows * nkb * 2;
            int s = 0;
            uint32_t ph = 0, issued = 0, last_ph[kRStages];
            for (int j = 0; j < nu; ++j) {
                if (!mbar_wait(&bars->empty[s], ph ^ 1, abort_flag, dev_err)) break;
                const int r0 = (u0 + j) * kRRows;
                uint8_t *st = ring + (size_t)s * sb;
                mbar_arrive_expect_tx(&bars->full[s], tx);
                for (int o = 0; o < nbox; ++o) tma_load_3d(st + o * kRBox, &tmq, &bars->full[s], 0, 2 * o, r0);
                tma_load_2d(st + (size_t)kRRows * K, &tms, &bars->full[s], 0, r0);
                issued |= 1u << s;
                last_ph[s] = ph;
                if (++s == kRStages) { s = 0; ph ^= 1; }
            }
            // copies issued last must land before shared memory is released
            for (int i = 0; i < kRStages; ++i)
                if (issued & (1u << i)) {
                    const long long t0 = clock64();
                    while (!mbar_try_wait(&bars->full[i], last_ph[i]))
                        if (clock64() - t0 > kWaitBudgetCycles) break;
                }
        }
        __syncwarp();
        pdl_trigger();
        return;
    }

    // ---------------------------------------------------- consumers
    pdl_trigger();
    pdl_wait();
    stage_x_rows<XT, kMode>(p, xs, (int)threadIdx.x - 32, kRW * 32);
    named_bar_sync(1, kRW * 32);

    const int cw = warp - 1;
    const int g = lane >> 2, t = lane & 3;
    // byte offsets of lane (g, t)'s 8 bytes for the 8 blocks of a box: line L = 2g +
    // (block / 4), 16-byte unit (block % 4) * 2 + t / 2 swizzled by L mod 8
    uint32_t off[8];
#pragma unroll
    for (int b8 = 0; b8 < 8; ++b8) {
        const uint32_t L = 2 * g + (b8 >> 2);
        const uint32_t unit = (uint32_t)((b8 & 3) * 2 + (t >> 1));
        off[b8] = L * 128 + ((unit ^ (L & 7)) << 4) + ((t & 1) << 3);
    }
    const uint4 *xg = xs + g * 4 + t;                 // chunk (b, g, t) = xg[b * R * 4]
    bool alive = true;
    for (int k = 0, j = cw; j < nu && alive; ++k, j += kRW) {
        const int s = cw + kRW * (k & 1);
        const uint32_t ph = (uint32_t)(k >> 1) & 1u;
        alive = warp_wait_all(&bars->full[s], ph, abort_flag, dev_err);
        if (!alive) break;
        const uint8_t *st = ring + (size_t)s * sb;
        const __half *sc = reinterpret_cast<const __half *>(st + (size_t)kRRows * K);
        const __half *sc0 = sc + (2 * t) * nkb, *sc1 = sc0 + nkb;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int o = 0; o < nbox; ++o) {
            const uint8_t *bx = st + o * kRBox;
            const uint4 s0v = *reinterpret_cast<const uint4 *>(sc0 + 8 * o);   // blocks 8o .. 8o+7, row 2t
            const uint4 s1v = *reinterpret_cast<const uint4 *>(sc1 + 8 * o);   // row 2t + 1
            const uint32_t s0w[4] = {s0v.x, s0v.y, s0v.z, s0v.w}, s1w[4] = {s1v.x, s1v.y, s1v.z, s1v.w};
#pragma unroll
            for (int b8 = 0; b8 < 8; ++b8) {
                const int b = 8 * o + b8;
                const uint2 w = *reinterpret_cast<const uint2 *>(bx + off[b8]);
                const uint4 xa = xg[(size_t)b * R * 4];
                uint4 xb = make_uint4(0u, 0u, 0u, 0u);
                if constexpr (R == 16) xb = xg[(size_t)b * R * 4 + 32];
                __half2 l0, h0, l1, h1;
                q8_to_half2x2(w.x, l0, h0);
                q8_to_half2x2(w.y, l1, h1);
                float d[4];
                {
                    const uint32_t a[4] = {xa.x, xb.x, xa.y, xb.y};
                    mma16816z(d, a, h2_as_u32(l0), h2_as_u32(h0));
                }
                {
                    const uint32_t a[4] = {xa.z, xb.z, xa.w, xb.w};
                    mma16816a(d, a, h2_as_u32(l1), h2_as_u32(h1));
                }
                const uint32_t sw0 = s0w[b8 >> 1], sw1 = s1w[b8 >> 1];
                const float f0 = __half2float(__ushort_as_half((unsigned short)((b8 & 1) ? (sw0 >> 16) : (sw0 & 0xffffu))));
                const float f1 = __half2float(__ushort_as_half((unsigned short)((b8 & 1) ? (sw1 >> 16) : (sw1 & 0xffffu))));
                if constexpr (kMode == kX32) {
                    acc[0] = fmaf(d[0] + d[2], f0, acc[0]);
                    acc[1] = fmaf(d[1] + d[3], f1, acc[1]);
                } else {
                    acc[0] = fmaf(d[0], f0, acc[0]);
                    acc[1] = fmaf(d[1], f1, acc[1]);
                    if constexpr (kMode == kX16W) {
                        acc[2] = fmaf(d[2], f0, acc[2]);
                        acc[3] = fmaf(d[3], f1, acc[3]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->empty[s]);   // stage consumed: the producer may refill it
        const int row = (u0 + j) * kRRows + 2 * t;
        store_one<YT, EPI, kQKV>(p, row, g, acc[0]);
        store_one<YT, EPI, kQKV>(p, row + 1, g, acc[1]);
        if constexpr (kMode == kX16W) {
            store_one<YT, EPI, kQKV>(p, row, g + 8, acc[2]);
            store_one<YT, EPI, kQKV>(p, row + 1, g + 8, acc[3]);
        }
    }
}

// Weights as a 3-D tensor [N][K/128][128] (bytes) read in [8][2][128] boxes with the
// 128-byte swizzle; scales as a 2-D tensor [N][K/32] (u16) read in [8][K/32] boxes.
bool make_rows_maps(const GemvArgs &a, CUtensorMap *tmq, CUtensorMap *tms) {
    PFN_encodeTiled enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t qd[3] = {128, (cuuint64_t)a.K / 128, (cuuint64_t)a.N};
    const cuuint64_t qstr[2] = {128, (cuuint64_t)a.K};
    const cuuint32_t qbox[3] = {128, 2, kRRows};
    const cuuint32_t es[3] = {1, 1, 1};
    if (enc(tmq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(a.qs), qd, qstr, qbox, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    const cuuint64_t sd[2] = {(cuuint64_t)a.K / 32, (cuuint64_t)a.N};
    const cuuint64_t sstr[1] = {(cuuint64_t)a.K / 16};
    const cuuint32_t sbox[2] = {(cuuint32_t)a.K / 32, kRRows};
    return enc(tms, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<__half *>(a.scales), sd, sstr, sbox, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename XT, typename YT, int EPI, bool kQKV, int kMode>
cudaError_t launch_rows_t(const GemvArgs &a, const CUtensorMap &tmq, const CUtensorMap &tms, int num_sms,
                          int *dev_err, cudaStream_t st, bool pdl) {
    auto fn = q8_gemv_rows_kernel<XT, YT, EPI, kQKV, kMode>;
    const size_t smem = rows_smem(kRMaxK, kMode);
    static std::once_flag once;
    static cudaError_t once_status;
    if (cudaError_t e = run_once(once, once_status, [&] {
            return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        }))
        return e;
    const int units = (a.N + kRRows - 1) / kRRows;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(units < num_sms ? units : num_sms);
    cfg.blockDim = dim3(kRThreads);
    cfg.dynamicSmemBytes = rows_smem(a.K, kMode);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, tmq, tms, a, dev_err);
}

template <typename XT, typename YT, int EPI, bool kQKV>
cudaError_t launch_rows_mode(const GemvArgs &a, bool x_split, const CUtensorMap &tmq, const CUtensorMap &tms,
                             int num_sms, int *dev_err, cudaStream_t st, bool pdl) {
    if (x_split) return launch_rows_t<float, YT, EPI, kQKV, kX32>(a, tmq, tms, num_sms, dev_err, st, pdl);
    return a.M > 8 ? launch_rows_t<XT, YT, EPI, kQKV, kX16W>(a, tmq, tms, num_sms, dev_err, st, pdl)
                   : launch_rows_t<XT, YT, EPI, kQKV, kX16>(a, tmq, tms, num_sms, dev_err, st, pdl);
}

}  // namespace

bool gemv_rows_ok(int M, int N, int K, bool x_f32) {
    if (M < 1 || N < 1 || K < 256 || K % 256 != 0 || K > kRMaxK) return false;
    return x_f32 ? M <= 8 : M <= 16;
}

bool gemv_use_rows(int M, int N, int K, bool x_f32_split) {
    static const int mode = [] {
        const char *e = getenv("MADI_GEMV_ROWS");
        return e ? (e[0] == '0' ? 0 : 1) : -1;
    }();
    if (mode != 1 || !gemv_rows_ok(M, N, K, x_f32_split)) return false;   // opt-in until measured
    return true;
}

cudaError_t launch_gemv_rows(const GemvArgs &a, bool x_f32, bool y_f32, int epi, bool qkv, int num_sms,
                             int *dev_err, cudaStream_t st, bool pdl, bool x_r16) {
    if (x_r16 && !x_f32) return cudaErrorInvalidValue;
    const bool split = x_f32 && !x_r16;
    if (!gemv_rows_ok(a.M, a.N, a.K, split)) return cudaErrorInvalidValue;
    CUtensorMap tmq, tms;
    if (!make_rows_maps(a, &tmq, &tms)) return cudaErrorNotSupported;
    if (qkv) return launch_rows_mode<float, float, kEpiNone, true>(a, split, tmq, tms, num_sms, dev_err, st, pdl);
#define MADI_ROWS_CASE(XT, YT)                                                                                    \
    switch (epi) {                                                                                                \
        case kEpiNone: return launch_rows_mode<XT, YT, kEpiNone, false>(a, split, tmq, tms, num_sms, dev_err, st, pdl); \
        case kEpiBias: return launch_rows_mode<XT, YT, kEpiBias, false>(a, split, tmq, tms, num_sms, dev_err, st, pdl); \
        case kEpiBiasGelu:                                                                                        \
            return launch_rows_mode<XT, YT, kEpiBiasGelu, false>(a, split, tmq, tms, num_sms, dev_err, st, pdl);  \
        case kEpiBiasRes:                                                                                         \
            return launch_rows_mode<XT, YT, kEpiBiasRes, false>(a, split, tmq, tms, num_sms, dev_err, st, pdl);   \
        default: return cudaErrorInvalidValue;                                                                    \
    }
    if (x_f32 && y_f32) { MADI_ROWS_CASE(float, float) }
    if (x_f32) { MADI_ROWS_CASE(float, __half) }
    if (y_f32) { MADI_ROWS_CASE(__half, float) }
    MADI_ROWS_CASE(__half, __half)
#undef MADI_ROWS_CASE
}

}  // namespace madi
