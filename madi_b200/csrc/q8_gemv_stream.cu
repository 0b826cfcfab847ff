// q8_gemv_stream.cu -- variant (b) for LARGE N (the vocab head): a persistent,
// TMA-streamed Q8_0 skinny GEMM, M <= 8.
//
// Same arithmetic as q8_gemv.cu (exact int8 -> f16, f32 per-block scale, f32
// activations split into f16 hi + lo, mma.sync m16n8k16 with f32 accumulation,
// graph_helpers.metal:320-352 semantics); different data movement:
//   * the unit of work is a 16-row tile: 16 x K int8 weights + 16 x K/32 f16
//     scales.  A producer lane fetches a tile into one ring stage with tiled TMA:
//     K/256 boxes of [16 rows][2][128 B] with the 128-byte swizzle (the weights
//     viewed as [N][K/128][128]) and one [16][K/32] box of scales.  Rows past N
//     arrive zero-filled;
//   * 16 consumer warps form two groups of 8 that take alternate tiles (four
//     warps per scheduler hide the MMA and shared-memory latencies); inside a
//     group, warp w takes the 32-blocks kb = w, w + 8, w + 16, ...  With kb mod 8
//     fixed per warp a lane's fragment address inside a box is a constant, and
//     the swizzle places the four rows a half-warp reads in four different bank
//     groups (conflict-free 8-byte loads);
//   * a group's eight [16 x 8] partial results meet in shared memory
//     (double-buffered); the group's warp (tile mod 8) adds them in warp order --
//     a fixed order, so results are run-to-run identical -- and runs the epilogue;
//   * CTAs are persistent (one per SM); the producer starts before
//     griddepcontrol.wait (weights do not depend on the previous kernel).
// Requirements (gemv_stream_ok + runtime): K % 256 == 0, K <= 8192, 16-byte
// aligned qs and scales, x staging plus >= 4 stages fit in shared memory.
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"

namespace madi {
namespace {

constexpr int kGroupWarps = 8;                           // one tile's consumers
constexpr int kGroups = 2;
constexpr int kConsumers = kGroupWarps * kGroups;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kTileRows = 16;
constexpr int kMaxStages = 8;
constexpr int kMinStages = 4;
constexpr int kBoxBytes = kTileRows * 256;               // one [16][2][128 B] weight box
constexpr size_t kRedBytes = (size_t)kGroups * 2 * kGroupWarps * 32 * 16;   // per group: 2 tiles x 8 warps x 32 lanes x float4
constexpr size_t kSmemBudget = 227 * 1024;

struct __align__(8) StreamBars {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    int abort;
};

// One stage: the K/256 weight boxes back to back (16 x K bytes), then the
// 16 x K/32 scales; rounded to 1 KB so every stage starts on the swizzle period.
__host__ __device__ constexpr size_t stage_bytes(int K) {
    return ((size_t)kTileRows * K + (size_t)kTileRows * (K / 32) * 2 + 1023) & ~size_t(1023);
}
__host__ __device__ constexpr size_t x_bytes(int M, int K, bool x_f32) { return (size_t)M * K * (x_f32 ? 4 : 2); }
__host__ __device__ constexpr size_t fixed_bytes(int M, int K, bool x_f32) {
    return 1024 + x_bytes(M, K, x_f32) + kRedBytes + sizeof(StreamBars);
}

int stage_count(int M, int K, bool x_f32) {
    const size_t used = fixed_bytes(M, K, x_f32);
    if (used >= kSmemBudget) return 0;
    size_t n = (kSmemBudget - used) / stage_bytes(K);
    if (n > kMaxStages) n = kMaxStages;
    return (int)(n & ~size_t(1));   // even: stage s always serves the same group
}

MADI_DEV void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T> MADI_DEV float s_to_f32(T v);
template <> MADI_DEV float s_to_f32<float>(float v) { return v; }
template <> MADI_DEV float s_to_f32<__half>(__half v) { return __half2float(v); }
template <typename T> MADI_DEV T s_from_f32(float v);
template <> MADI_DEV float s_from_f32<float>(float v) { return v; }
template <> MADI_DEV __half s_from_f32<__half>(float v) { return __float2half_rn(v); }

// Byte offset, inside one weight box, of the 8 bytes lane t reads from tile row
// `row` for a 32-block with kb mod 8 == w.  Row position P = (kb mod 8) x 32 + 8t
// lies in 128-byte line L = 2 row + (kb / 4 mod 2); the swizzle XORs the 16-byte
// unit index with L mod 8.
MADI_DEV uint32_t frag_offset(int row, int w, int t) {
    const int L = 2 * row + ((w >> 2) & 1);
    const int unit = ((w & 3) << 1) | (t >> 1);
    return (uint32_t)(L * 128 + ((unit ^ (L & 7)) << 4) + ((t & 1) << 3));
}

template <typename XT, typename YT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    q8_gemv_stream_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tms,
                          const GemvArgs p, int stages, int *dev_err) {
    constexpr bool kSplit = sizeof(XT) == 4;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int M = p.M, K = p.K, N = p.N;
    const int nkb = K >> 5;
    const size_t sb = stage_bytes(K);
    uint8_t *ring = smem;
    uint8_t *xs = smem + (size_t)stages * sb;
    float4 *red = reinterpret_cast<float4 *>(xs + x_bytes(M, K, kSplit));
    StreamBars *bars = reinterpret_cast<StreamBars *>(reinterpret_cast<uint8_t *>(red) + kRedBytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = (N + kTileRows - 1) / kTileRows;
    volatile int *abort_flag = &bars->abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], kGroupWarps);
        }
        bars->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------ producer: one stage = one 16-row tile
        if (lane == 0) {
            tma_prefetch_desc(&tmq);
            tma_prefetch_desc(&tms);
            const uint32_t tx = (uint32_t)(K / 256) * kBoxBytes + (uint32_t)kTileRows * nkb * 2;
            int s = 0;
            uint32_t ph = 0;
            uint32_t issued = 0, last_ph[kMaxStages];
            for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                if (!mbar_wait(&bars->empty[s], ph ^ 1, abort_flag, dev_err)) break;
                const int r0 = tile * kTileRows;
                uint8_t *st = ring + (size_t)s * sb;
                mbar_arrive_expect_tx(&bars->full[s], tx);
                for (int o = 0; o < K / 256; ++o) tma_load_3d(st + o * kBoxBytes, &tmq, &bars->full[s], 0, 2 * o, r0);
                tma_load_2d(st + (size_t)kTileRows * K, &tms, &bars->full[s], 0, r0);
                issued |= 1u << s;
                last_ph[s] = ph;
                if (++s == stages) { s = 0; ph ^= 1; }
            }
            // copies issued last must land before shared memory is released
            for (int i = 0; i < stages; ++i)
                if (issued & (1u << i)) {
                    const long long t0 = clock64();
                    while (!mbar_try_wait(&bars->full[i], last_ph[i]))
                        if (clock64() - t0 > kWaitBudgetCycles) break;
                }
        }
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        __syncwarp();
        return;
    }

    // ---------------------------------------------------- consumers
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // stage x once per CTA in fragment order: slot (kb, s, m, t) holds
    // x[m][kb*32 + 8t + 4s + 0..3] as f16 hi (and, for f32 x, f16 lo) pairs;
    // loads go out in batches of 8 per thread so the L2 round trips overlap
    {
        constexpr int B = 8;
        const int ct = threadIdx.x - 32, nct = kConsumers * 32;
        const int nq = M * K / 4;
        for (int base = ct; base < nq; base += B * nct) {
            float v[B][4];
#pragma unroll
            for (int j = 0; j < B; ++j) {
                const int i = base + j * nct;
                if (i < nq) {
                    if constexpr (kSplit) {
                        const float4 f = __ldg(reinterpret_cast<const float4 *>(p.x) + i);
                        v[j][0] = f.x; v[j][1] = f.y; v[j][2] = f.z; v[j][3] = f.w;
                    } else {
                        const uint2 u = __ldg(reinterpret_cast<const uint2 *>(p.x) + i);
                        const __half2 h0 = *reinterpret_cast<const __half2 *>(&u.x);
                        const __half2 h1 = *reinterpret_cast<const __half2 *>(&u.y);
                        v[j][0] = __low2float(h0); v[j][1] = __high2float(h0);
                        v[j][2] = __low2float(h1); v[j][3] = __high2float(h1);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < B; ++j) {
                const int i = base + j * nct;
                if (i < nq) {
                    const int m = (4 * i) / K, k = (4 * i) % K;
                    const int kb = k >> 5, t = (k & 31) >> 3, s = (k & 7) >> 2;
                    const int slot = ((kb * 2 + s) * M + m) * 4 + t;
                    const __half2 h01 = __floats2half2_rn(v[j][0], v[j][1]), h23 = __floats2half2_rn(v[j][2], v[j][3]);
                    if constexpr (kSplit) {
                        const __half2 l01 = __floats2half2_rn(v[j][0] - __low2float(h01), v[j][1] - __high2float(h01));
                        const __half2 l23 = __floats2half2_rn(v[j][2] - __low2float(h23), v[j][3] - __high2float(h23));
                        reinterpret_cast<uint4 *>(xs)[slot] =
                            make_uint4(h2_as_u32(h01), h2_as_u32(h23), h2_as_u32(l01), h2_as_u32(l23));
                    } else {
                        reinterpret_cast<uint2 *>(xs)[slot] = make_uint2(h2_as_u32(h01), h2_as_u32(h23));
                    }
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");   // all consumers
    }

    const int cw = warp - 1;
    const int grp = cw / kGroupWarps, wg = cw % kGroupWarps;
    const int g8 = lane >> 2, t = lane & 3;
    const bool gval = g8 < M;
    const int nki = nkb >> 3;                          // 32-blocks per warp per tile
    const uint32_t off0 = frag_offset(g8, wg, t), off1 = frag_offset(g8 + 8, wg, t);
    const int xstep = 16 * M * 4;                      // x slots per i (8 blocks x 2 halves x M x 4)
    const int xbase = (wg * 2 * M + g8) * 4 + t;       // slot of (kb = wg, s = 0, m = g8, t)
    float4 *red_g = red + (size_t)grp * 2 * kGroupWarps * 32;
    bool alive = true;
    // Group g takes the CTA's tiles n = g, g + 2, ...; the stage count is even, so a
    // stage's previous round belongs to the same group and was waited for by every
    // warp of it (parity waits stay unambiguous).  Every warp of a group runs the
    // same tiles, so the group's named barrier is met by its 256 threads each time,
    // also after a bounded wait gave up.
    for (int n = grp, j = 0; blockIdx.x + n * gridDim.x < tiles; n += kGroups, ++j) {
        const int tile = blockIdx.x + n * gridDim.x;
        const int s = n % stages;
        const uint32_t ph = (uint32_t)(n / stages) & 1u;
        if (alive) alive = warp_wait_all(&bars->full[s], ph, abort_flag, dev_err);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (alive) {
            const uint8_t *st = ring + (size_t)s * sb;
            const __half *sc = reinterpret_cast<const __half *>(st + (size_t)kTileRows * K);
            const __half *s0p = sc + g8 * nkb + wg, *s1p = s0p + 8 * nkb;
#pragma unroll 4
            for (int i = 0; i < nki; ++i) {
                const uint2 wa = *reinterpret_cast<const uint2 *>(st + off0 + i * kBoxBytes);
                const uint2 wb = *reinterpret_cast<const uint2 *>(st + off1 + i * kBoxBytes);
                float bh[4] = {0.f, 0.f, 0.f, 0.f}, bl[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int sp = 0; sp < 2; ++sp) {
                    __half2 a_lo0, a_hi0, a_lo1, a_hi1;
                    q8_to_half2x2(sp == 0 ? wa.x : wa.y, a_lo0, a_hi0);
                    q8_to_half2x2(sp == 0 ? wb.x : wb.y, a_lo1, a_hi1);
                    const uint32_t a[4] = {h2_as_u32(a_lo0), h2_as_u32(a_lo1), h2_as_u32(a_hi0), h2_as_u32(a_hi1)};
                    const int slot = xbase + i * xstep + sp * M * 4;
                    if constexpr (kSplit) {
                        const uint4 xv = gval ? reinterpret_cast<const uint4 *>(xs)[slot] : make_uint4(0u, 0u, 0u, 0u);
                        mma16816(bh, a, xv.x, xv.y);
                        mma16816(bl, a, xv.z, xv.w);
                    } else {
                        const uint2 xv = gval ? reinterpret_cast<const uint2 *>(xs)[slot] : make_uint2(0u, 0u);
                        mma16816(sp == 0 ? bh : bl, a, xv.x, xv.y);
                    }
                }
                const float f0 = __half2float(s0p[8 * i]);
                const float f1 = __half2float(s1p[8 * i]);
                acc[0] = fmaf(bh[0] + bl[0], f0, acc[0]);
                acc[1] = fmaf(bh[1] + bl[1], f0, acc[1]);
                acc[2] = fmaf(bh[2] + bl[2], f1, acc[2]);
                acc[3] = fmaf(bh[3] + bl[3], f1, acc[3]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->empty[s]);   // stage consumed: the producer may refill it
        float4 *rb = red_g + (size_t)(j & 1) * kGroupWarps * 32;
        rb[wg * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        asm volatile("bar.sync %0, %1;" ::"r"(2 + grp), "r"(kGroupWarps * 32) : "memory");
        // The reducer of the group's tile j reads buffer j & 1 before it reaches the
        // group barrier of tile j + 1, and tile j + 2 rewrites that buffer only after it.
        if (wg != (j & (kGroupWarps - 1)) || !alive) continue;
        float v4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < kGroupWarps; ++w) {
            const float4 q = rb[w * 32 + lane];
            v4[0] += q.x; v4[1] += q.y; v4[2] += q.z; v4[3] += q.w;
        }
        // v4[0..1] = (row g8, tokens 2t, 2t+1), v4[2..3] = (row g8 + 8, ...)
        const int row0 = tile * kTileRows + g8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = (i < 2) ? row0 : row0 + 8;
            const int tok = 2 * t + (i & 1);
            if (row >= N || tok >= M) continue;
            float v = v4[i];
            float bb = 0.f;
            if constexpr (EPI != kEpiNone)
                bb = p.bias_f16 ? __half2float(reinterpret_cast<const __half *>(p.bias)[row])
                                : reinterpret_cast<const float *>(p.bias)[row];
            const size_t o = (size_t)tok * N + row;
            if constexpr (EPI == kEpiBias) v = v + bb;
            if constexpr (EPI == kEpiBiasGelu) v = gelu_erf(v + bb);
            if constexpr (EPI == kEpiBiasRes) v = s_to_f32(reinterpret_cast<const YT *>(p.residual)[o]) + v + bb;
            reinterpret_cast<YT *>(p.y)[o] = s_from_f32<YT>(v);
        }
    }
}

// Weights as a 3-D tensor [N][K/128][128] (bytes) read in [16][2][128] boxes with
// the 128-byte swizzle; scales as a 2-D tensor [N][K/32] (u16) read in [16][K/32]
// boxes.  Out-of-range rows are zero-filled.
bool make_stream_maps(const GemvArgs &a, CUtensorMap *tmq, CUtensorMap *tms) {
    PFN_encodeTiled enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t qd[3] = {128, (cuuint64_t)a.K / 128, (cuuint64_t)a.N};
    const cuuint64_t qstr[2] = {128, (cuuint64_t)a.K};
    const cuuint32_t qbox[3] = {128, 2, kTileRows};
    const cuuint32_t es[3] = {1, 1, 1};
    if (enc(tmq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(a.qs), qd, qstr, qbox, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    const cuuint64_t sd[2] = {(cuuint64_t)a.K / 32, (cuuint64_t)a.N};
    const cuuint64_t sstr[1] = {(cuuint64_t)a.K / 16};
    const cuuint32_t sbox[2] = {(cuuint32_t)a.K / 32, kTileRows};
    return enc(tms, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<__half *>(a.scales), sd, sstr, sbox, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename XT, typename YT, int EPI>
cudaError_t launch_stream_one(const GemvArgs &a, const CUtensorMap &tmq, const CUtensorMap &tms, int num_sms,
                              int *dev_err, cudaStream_t st, bool pdl) {
    const bool xf32 = sizeof(XT) == 4;
    const int stages = stage_count(a.M, a.K, xf32);
    const size_t smem = fixed_bytes(a.M, a.K, xf32) + (size_t)stages * stage_bytes(a.K);
    auto fn = q8_gemv_stream_kernel<XT, YT, EPI>;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    const int tiles = (a.N + kTileRows - 1) / kTileRows;
    const int grid = tiles < num_sms ? tiles : num_sms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, tmq, tms, a, stages, dev_err);
}

}  // namespace

// Large N only (at least kMinTilesPerSm 16-row tiles per SM), K a multiple of 256
// (whole weight boxes; every scale row K/16 bytes, a multiple of 16 as the tensor
// map's strides require) and at most 8192 (one scale box per tile), and room in
// shared memory for x, the partial sums and >= kMinStages tiles.
bool gemv_stream_ok(int M, int N, int K, bool x_f32, int num_sms) {
    constexpr int kMinTilesPerSm = 4;
    const long tiles = (N + kTileRows - 1) / kTileRows;
    if (K % 256 != 0 || K > 8192 || tiles < (long)kMinTilesPerSm * num_sms) return false;
    return stage_count(M, K, x_f32) >= kMinStages;
}

cudaError_t launch_gemv_stream(const GemvArgs &a, bool x_f32, bool y_f32, int epi, int num_sms, int *dev_err,
                               cudaStream_t st, bool pdl) {
    CUtensorMap tmq, tms;
    if (!make_stream_maps(a, &tmq, &tms)) return cudaErrorNotSupported;
#define MADI_STREAM_CASE(XT, YT)                                                                          \
    switch (epi) {                                                                                        \
        case kEpiNone: return launch_stream_one<XT, YT, kEpiNone>(a, tmq, tms, num_sms, dev_err, st, pdl);  \
        case kEpiBias: return launch_stream_one<XT, YT, kEpiBias>(a, tmq, tms, num_sms, dev_err, st, pdl);  \
        case kEpiBiasGelu:                                                                                \
            return launch_stream_one<XT, YT, kEpiBiasGelu>(a, tmq, tms, num_sms, dev_err, st, pdl);       \
        case kEpiBiasRes:                                                                                 \
            return launch_stream_one<XT, YT, kEpiBiasRes>(a, tmq, tms, num_sms, dev_err, st, pdl);        \
        default: return cudaErrorInvalidValue;                                                            \
    }
    if (x_f32 && y_f32) { MADI_STREAM_CASE(float, float) }
    if (x_f32 && !y_f32) { MADI_STREAM_CASE(float, __half) }
    if (!x_f32 && y_f32) { MADI_STREAM_CASE(__half, float) }
    MADI_STREAM_CASE(__half, __half)
#undef MADI_STREAM_CASE
}

}  // namespace madi
