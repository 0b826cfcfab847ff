// q8_gemv.cu -- variant (b): bandwidth-bound Q8_0 GEMV / skinny GEMM, M <= 8.
//
// Semantics (reference graph_helpers.metal:320-567, f32 throughout):
//   y[m][n] = epi( sum_kb s[n][kb] * sum_{k in kb} x[m][k] * q[n][k] )
// The int8 weights are converted to f16 EXACTLY (no scale folded in), the
// per-32-block scale is applied in f32 to each block's partial sum, and f32
// activations are split into two f16 halves (hi = f16(x), lo = f16(x - hi))
// so the products keep ~22 mantissa bits.  Accumulation is f32.
//
// Mapping onto the tensor cores (mma.sync m16n8k16, f16 in, f32 accumulate):
// the MMA "M" dimension is 16 weight rows, "N" is the 8 token slots, "K" walks
// one Q8 block (32) in two k16 steps.  Because a dot product does not care in
// which order its terms are summed, the MMA's k-slots are bound to physical k
// so that each lane reads 8 CONTIGUOUS int8 of a row per block:
//   lane (g = lane/4, t = lane%4) owns physical k = 8t .. 8t+7 of the block;
//   step s uses 8t+4s .. 8t+4s+3; A slots {2t,2t+1} <- k+0,1 and {2t+8,2t+9} <- k+2,3.
// The activations are staged per CTA in shared memory already permuted into
// that fragment order, so every B-fragment read is one conflict-free 8-byte load.
//
// Work split: a CTA is 8 warps, one 16-row tile each (128 rows).  A thread-
// block cluster of `cs` CTAs (1..16) shares the same 128 rows and splits K:
// CTA rank r streams K blocks [r*bpw, (r+1)*bpw) and stages only that slice of
// x.  The partial sums meet in the rank-0 CTA through distributed shared
// memory and are added in rank order (deterministic, no atomics, no global
// scratch).
//
// Streaming: a decode GEMV moves only a few MB, so it is latency-bound unless
// the whole matrix is in flight at once.  Each warp therefore requests ALL of
// its slice (bpw <= kMaxB blocks: 16 rows x bpw x 32 bytes) in one round, and
// does so before griddepcontrol.wait: the weights do not depend on the
// previous kernel, so under programmatic dependent launch they stream while
// that kernel drains.
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"

namespace cg = cooperative_groups;

namespace madi {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 16 * kWarps;   // weight rows per CTA
constexpr int kMaxB = 10;            // Q8 blocks a warp keeps in flight (one round)
constexpr int kMaxCluster = 16;      // non-portable cluster size, allowed on sm_100

// Predicated streaming load into registers the caller pre-set to zero.  No
// instruction consumes the value inside the asm, so all of a warp's loads are
// in flight together and the thread waits only at the MMA that uses them.
MADI_DEV void ldg_stream_u2_pred(uint2 &v, const void *p, bool pred) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %3, 0;\n\t"
        "@q ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];\n\t}"
        : "+r"(v.x), "+r"(v.y)
        : "l"(p), "r"((int)pred));
}

MADI_DEV void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T> MADI_DEV float to_f32(T v);
template <> MADI_DEV float to_f32<float>(float v) { return v; }
template <> MADI_DEV float to_f32<__half>(__half v) { return __half2float(v); }
template <typename T> MADI_DEV T from_f32(float v);
template <> MADI_DEV float from_f32<float>(float v) { return v; }
template <> MADI_DEV __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Stage x[m][k] for k in this CTA's slice [kb_begin*32, kb_end*32) into shared
// memory in fragment order: slot (lkb, s, m, t) holds x[m][(kb_begin+lkb)*32 +
// 8t + 4s + 0..3] as four f16.  Loads are issued in batches of 8 per thread so
// the L2 round trips overlap; they use the coherent L2 path (ld.global.cg)
// because under programmatic dependent launch x is written by a kernel whose
// lifetime overlaps this one's.
template <typename XT, bool kSplit>
MADI_DEV void stage_x(const XT *__restrict__ x, int M, int K, int kb_begin, int kb_end, uint2 *xf_hi,
                      uint2 *xf_lo) {
    constexpr int B = 8;
    const int qrow = (kb_end - kb_begin) * 8;   // quads of 4 elements per token row
    const int nq = M * qrow;
    for (int base = threadIdx.x; base < nq; base += B * kThreads) {
        float v[B][4];
#pragma unroll
        for (int j = 0; j < B; ++j) {
            const int i = base + j * kThreads;
            if (i < nq) {
                const int m = i / qrow, kq = i - m * qrow;
                const size_t off = (size_t)m * K + (size_t)kb_begin * 32 + 4 * kq;
                if constexpr (sizeof(XT) == 4) {
                    const float4 f = __ldcg(reinterpret_cast<const float4 *>(x + off));
                    v[j][0] = f.x; v[j][1] = f.y; v[j][2] = f.z; v[j][3] = f.w;
                } else {
                    const uint2 u = __ldcg(reinterpret_cast<const uint2 *>(x + off));
                    const __half2 h0 = *reinterpret_cast<const __half2 *>(&u.x);
                    const __half2 h1 = *reinterpret_cast<const __half2 *>(&u.y);
                    v[j][0] = __low2float(h0); v[j][1] = __high2float(h0);
                    v[j][2] = __low2float(h1); v[j][3] = __high2float(h1);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < B; ++j) {
            const int i = base + j * kThreads;
            if (i < nq) {
                const int m = i / qrow, kq = i - m * qrow;
                const int lkb = kq >> 3, t = (kq & 7) >> 1, s = kq & 1;
                const int slot = ((lkb * 2 + s) * M + m) * 4 + t;
                const __half2 h01 = __floats2half2_rn(v[j][0], v[j][1]), h23 = __floats2half2_rn(v[j][2], v[j][3]);
                xf_hi[slot] = make_uint2(h2_as_u32(h01), h2_as_u32(h23));
                if constexpr (kSplit) {
                    const __half2 l01 = __floats2half2_rn(v[j][0] - __low2float(h01), v[j][1] - __high2float(h01));
                    const __half2 l23 = __floats2half2_rn(v[j][2] - __low2float(h23), v[j][3] - __high2float(h23));
                    xf_lo[slot] = make_uint2(h2_as_u32(l01), h2_as_u32(l23));
                }
            }
        }
    }
}

template <typename XT, typename YT, int EPI, bool kQKV>
__global__ void __launch_bounds__(kThreads, 2) q8_gemv_kernel(const GemvArgs p) {
    constexpr bool kSplit = sizeof(XT) == 4;
    extern __shared__ __align__(16) uint8_t smem[];
    const int M = p.M, K = p.K, N = p.N, cs = p.ks;
    const int nkb = K >> 5;
    const int bpw = (nkb + cs - 1) / cs;                          // blocks per CTA (and per warp)
    const int rank = cs > 1 ? (int)(blockIdx.x % cs) : 0;        // cluster rank along x
    const int group = cs > 1 ? (int)(blockIdx.x / cs) : (int)blockIdx.x;
    const int kb_begin = min(nkb, rank * bpw);
    const int kb_end = min(nkb, kb_begin + bpw);
    const size_t slot_count = (size_t)(kb_end - kb_begin) * 8 * M;   // uint2 slots per half
    uint2 *xf_hi = reinterpret_cast<uint2 *>(smem);
    uint2 *xf_lo = xf_hi + slot_count;
    float4 *red = reinterpret_cast<float4 *>(smem + (size_t)bpw * 8 * 8 * (kSplit ? 16 : 8));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int row0 = group * kRows + warp * 16 + g, row1 = row0 + 8;
    const bool ok0 = row0 < N, ok1 = row1 < N;

    const int8_t *w0 = p.qs + (size_t)(ok0 ? row0 : 0) * K + 8 * t;
    const int8_t *w1 = p.qs + (size_t)(ok1 ? row1 : 0) * K + 8 * t;
    const __half *s0p = p.scales + (size_t)(ok0 ? row0 : 0) * nkb;
    const __half *s1p = p.scales + (size_t)(ok1 ? row1 : 0) * nkb;

    uint2 wa[kMaxB], wb[kMaxB];
    uint32_t sa[kMaxB], sb[kMaxB];     // raw f16 scale bits, converted at use
    auto load_round = [&](int kb0) {
#pragma unroll
        for (int u = 0; u < kMaxB; ++u) {
            const int kb = kb0 + u;
            const bool in = kb < kb_end;
            const int kbc = in ? kb : kb_begin;     // a valid address even when predicated off
            wa[u] = make_uint2(0u, 0u);
            wb[u] = make_uint2(0u, 0u);
            sa[u] = 0u;
            sb[u] = 0u;
            ldg_stream_u2_pred(wa[u], w0 + (size_t)kbc * 32, in && ok0);
            ldg_stream_u2_pred(wb[u], w1 + (size_t)kbc * 32, in && ok1);
            ldg_nc_u16_pred(sa[u], s0p + kbc, in && ok0);
            ldg_nc_u16_pred(sb[u], s1p + kbc, in && ok1);
        }
    };

    // the whole slice of weights first, before waiting on the kernel that produced x
    load_round(kb_begin);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    stage_x<XT, kSplit>(reinterpret_cast<const XT *>(p.x), M, K, kb_begin, kb_end, xf_hi, xf_lo);
    __syncthreads();

    const bool gval = g < M;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int kb0 = kb_begin; kb0 < kb_end; kb0 += kMaxB) {
        if (kb0 != kb_begin) load_round(kb0);   // only when a slice exceeds kMaxB blocks
#pragma unroll
        for (int u = 0; u < kMaxB; ++u) {
            const int kb = kb0 + u;
            if (kb >= kb_end) break;
            float blk[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                __half2 a_lo0, a_hi0, a_lo1, a_hi1;
                q8_to_half2x2(s == 0 ? wa[u].x : wa[u].y, a_lo0, a_hi0);
                q8_to_half2x2(s == 0 ? wb[u].x : wb[u].y, a_lo1, a_hi1);
                const uint32_t a[4] = {h2_as_u32(a_lo0), h2_as_u32(a_lo1), h2_as_u32(a_hi0), h2_as_u32(a_hi1)};
                const int slot = (((kb - kb_begin) * 2 + s) * M + g) * 4 + t;
                const uint2 bh = gval ? xf_hi[slot] : make_uint2(0u, 0u);
                mma16816(blk, a, bh.x, bh.y);
                if constexpr (kSplit) {
                    const uint2 bl = gval ? xf_lo[slot] : make_uint2(0u, 0u);
                    mma16816(blk, a, bl.x, bl.y);
                }
            }
            const float s0 = __half2float(__ushort_as_half((unsigned short)sa[u]));
            const float s1 = __half2float(__ushort_as_half((unsigned short)sb[u]));
            acc[0] = fmaf(blk[0], s0, acc[0]);
            acc[1] = fmaf(blk[1], s0, acc[1]);
            acc[2] = fmaf(blk[2], s1, acc[2]);
            acc[3] = fmaf(blk[3], s1, acc[3]);
        }
    }

    if (cs > 1) {
        // cross-CTA split-K: partials meet in the rank-0 CTA through DSMEM
        red[warp * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        if (rank == 0) {
            for (int j = 1; j < cs; ++j) {
                const float4 o = cluster.map_shared_rank(red, j)[warp * 32 + lane];
                acc[0] += o.x; acc[1] += o.y; acc[2] += o.z; acc[3] += o.w;
            }
        }
        cluster.sync();   // remote shared memory stays alive until it has been read
        if (rank != 0) return;
    }

    // C fragment: acc[0..1] = (row0, tokens 2t, 2t+1), acc[2..3] = (row1, ...)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = (i < 2) ? row0 : row1;
        const int tok = 2 * t + (i & 1);
        if (row >= N || tok >= M) continue;
        float v = acc[i];
        if constexpr (kQKV) {
            const int D = p.D;
            if (row < D) {
                reinterpret_cast<float *>(p.y)[(size_t)tok * D + row] = v + p.qb[row];
            } else {
                const size_t base = (size_t)tok * p.cache_stride + (size_t)p.pos[tok] * D;
                if (row < 2 * D) p.kc[base + (row - D)] = v;
                else p.vc[base + (row - 2 * D)] = v + p.vb[row - 2 * D];
            }
        } else {
            float b = 0.f;
            if constexpr (EPI != kEpiNone)
                b = p.bias_f16 ? __half2float(reinterpret_cast<const __half *>(p.bias)[row])
                               : reinterpret_cast<const float *>(p.bias)[row];
            const size_t o = (size_t)tok * N + row;
            if constexpr (EPI == kEpiBias) v = v + b;
            if constexpr (EPI == kEpiBiasGelu) v = gelu_erf(v + b);
            if constexpr (EPI == kEpiBiasRes) v = to_f32(reinterpret_cast<const YT *>(p.residual)[o]) + v + b;
            reinterpret_cast<YT *>(p.y)[o] = from_f32<YT>(v);
        }
    }
}

template <typename XT, typename YT, int EPI, bool kQKV>
cudaError_t launch_one(const GemvArgs &a, cudaStream_t st, bool pdl) {
    const size_t smem = gemv_smem_bytes(a.M, a.K, a.ks, sizeof(XT) == 4);
    auto fn = q8_gemv_kernel<XT, YT, EPI, kQKV>;
    // raise the dynamic shared-memory cap once per instantiation (to the
    // largest ever needed), so a launch inside a graph capture is only a launch
    static size_t smem_cap = 48 * 1024;
    static bool cluster_attr = false;
    static std::mutex mu;                 // host threads share the two attributes
    {
        std::lock_guard<std::mutex> lk(mu);
        if (smem > smem_cap) {
            cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            smem_cap = smem;
        }
        if (!cluster_attr && a.ks > 8) {
            cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return e;
            cluster_attr = true;
        }
    }
    const int groups = (a.N + kRows - 1) / kRows;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(groups * a.ks);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    ++na;
    if (a.ks > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = a.ks;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace

// Cluster size (cross-CTA K split): about kMaxB Q8 blocks per warp so a slice
// is one round of loads, at most 16 CTAs per cluster -- then halved while the
// grid would exceed ~6 CTAs per SM (large N has parallelism in rows already).
// Measured on B200 (decode shapes, M = 1 and 8, under PDL): K = 1280 -> 4,
// K = 5120 -> 16, vocab head (N = 51866) -> 2.
int gemv_pick_ks(int N, int K, int num_sms) {
    const int groups = (N + kRows - 1) / kRows;
    const int nkb = K / 32;
    int cs = (nkb + kMaxB - 1) / kMaxB;
    if (cs < 1) cs = 1;
    if (cs > kMaxCluster) cs = kMaxCluster;
    while (cs > 1 && groups * cs > 6 * num_sms) cs = (cs + 1) / 2;
    return cs;
}

size_t gemv_smem_bytes(int M, int K, int cs, bool x_f32) {
    const int nkb = K / 32;
    const int bpw = (nkb + cs - 1) / cs;
    (void)M;
    // x slice sized for the maximum 8 token slots so every launch of an
    // instantiation fits the same cap, plus the partial-sum exchange area
    return (size_t)bpw * 8 * 8 * (x_f32 ? 16 : 8) + (size_t)kThreads * 16;
}

cudaError_t launch_gemv(const GemvArgs &a, bool x_f32, bool y_f32, int epi, bool qkv, cudaStream_t st, bool pdl) {
    if (qkv) return x_f32 ? launch_one<float, float, kEpiNone, true>(a, st, pdl)
                          : launch_one<__half, float, kEpiNone, true>(a, st, pdl);
#define MADI_GEMV_CASE(XT, YT)                                                  \
    switch (epi) {                                                              \
        case kEpiNone: return launch_one<XT, YT, kEpiNone, false>(a, st, pdl);  \
        case kEpiBias: return launch_one<XT, YT, kEpiBias, false>(a, st, pdl);  \
        case kEpiBiasGelu: return launch_one<XT, YT, kEpiBiasGelu, false>(a, st, pdl); \
        case kEpiBiasRes: return launch_one<XT, YT, kEpiBiasRes, false>(a, st, pdl);   \
        default: return cudaErrorInvalidValue;                                  \
    }
    if (x_f32 && y_f32) { MADI_GEMV_CASE(float, float) }
    if (x_f32 && !y_f32) { MADI_GEMV_CASE(float, __half) }
    if (!x_f32 && y_f32) { MADI_GEMV_CASE(__half, float) }
    MADI_GEMV_CASE(__half, __half)
#undef MADI_GEMV_CASE
}

}  // namespace madi
