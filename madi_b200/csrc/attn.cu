// attn.cu -- decoder attention beside the Q8 projections (decoder_ops.metal:81-530).
//
//   gpu_attention                   self-attention of one query token per slot over
//                                   the f32 KV cache rows 0..pos (pos read on the
//                                   device)                                        (:81-149)
//   flash_cross_attn[_f16kv]        cross-attention of one query token per slot over
//                                   `seqlen` encoder positions, f32 or f16 K/V,
//                                   optional normalised scores                     (:191-325)
//   flash_cross_attn_f16kv_batched  the same for B slots, each with its own K/V    (:459-531)
//   flash_cross_attn_split/_reduce  the two-pass form with caller-owned partials   (:327-457)
//
// Scores are q.k * rsqrt(head_dim); softmax as exp2((s - max) * log2 e); head_dim 64.
//
// B200 layout of the fused attention (cross- and self-): one thread-block cluster
// of `ns` CTAs (<= 8) per (slot, head).  CTA c TMA-loads its chunk of keys and
// values ([csz][64] boxes of its kv head) into shared memory, computes its partial
// flash result -- local max m, exp-sum s and unnormalised o = sum e*v -- and
// pushes (m, s, o) into rank 0's shared memory; rank 0 recombines them by
// log-sum-exp (the reference's flash_cross_attn_reduce arithmetic) and writes the
// output.  No global scratch and one launch, with (slots x heads x ns) CTAs
// streaming K/V in parallel.  The cross-attention K/V is the decode step's largest
// read at 8 slots (2 x 1500 x 1280 f16 per slot per layer): the kernel is HBM-bound.
#include <algorithm>
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace cg = cooperative_groups;

namespace madi {
namespace {

constexpr int kHd = 64;
constexpr int kThr = 256;
constexpr float kLog2e = 1.4426950408889634f;

MADI_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
MADI_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// Block-wide max / sum over 256 threads, result in every thread.  `s8` holds
// the 8 warp partials; the trailing barrier lets the caller reuse it.
MADI_DEV float block_max(float v, float *s8) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) s8[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = s8[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) r = fmaxf(r, s8[i]);
    __syncthreads();
    return r;
}
MADI_DEV float block_sum(float v, float *s8) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) s8[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) r += s8[i];
    __syncthreads();
    return r;
}

template <typename T> MADI_DEV float4 ld4(const T *p);
template <> MADI_DEV float4 ld4<float>(const float *p) { return *reinterpret_cast<const float4 *>(p); }
template <> MADI_DEV float4 ld4<__half>(const __half *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
template <typename T> MADI_DEV float2 ld2(const T *p);
template <> MADI_DEV float2 ld2<float>(const float *p) { return *reinterpret_cast<const float2 *>(p); }
template <> MADI_DEV float2 ld2<__half>(const __half *p) {
    return __half22float2(*reinterpret_cast<const __half2 *>(p));
}

// raw[k] = q_h . K[k] * rsqrt(64) for k in [0, n); a half-warp per key.
template <typename KV>
MADI_DEV void scores_of(const float *qh, const KV *kb, int kvd, int n, float *raw) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hw = lane >> 4, li = lane & 15;
    const float4 qv = make_float4(qh[4 * li], qh[4 * li + 1], qh[4 * li + 2], qh[4 * li + 3]);
    const float rsq = rsqrtf((float)kHd);
    for (int k0 = warp * 2; k0 < n; k0 += 16) {      // warp-uniform bound: all lanes shuffle
        const int k = k0 + hw;
        float d = 0.f;
        if (k < n) {
            const float4 kv = ld4(kb + (size_t)k * kvd + 4 * li);
            d = qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
        }
        d += __shfl_xor_sync(0xffffffffu, d, 8);
        d += __shfl_xor_sync(0xffffffffu, d, 4);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        if (li == 0 && k < n) raw[k] = d * rsq;
    }
}

// o[d] = sum_k w[k] * V[k][d] for d < 64, returned in threads 0..63 (a warp per
// key, lanes over dims; the 8 warp sums are added in warp order).
template <typename KV>
MADI_DEV float pv_of(const float *w, const KV *vb, int kvd, int n, float (*red)[kHd]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float a0 = 0.f, a1 = 0.f;
    for (int k = warp; k < n; k += 8) {
        const float2 v = ld2(vb + (size_t)k * kvd + 2 * lane);
        a0 = fmaf(w[k], v.x, a0);
        a1 = fmaf(w[k], v.y, a1);
    }
    red[warp][2 * lane] = a0;
    red[warp][2 * lane + 1] = a1;
    __syncthreads();
    float o = 0.f;
    if (threadIdx.x < kHd) {
#pragma unroll
        for (int w8 = 0; w8 < 8; ++w8) o += red[w8][threadIdx.x];
    }
    return o;
}

// ---------------------------------------------------------------- fused attention
// grid (ns, heads, slots), cluster (ns, 1, 1) when ns > 1.  K and V are viewed as
// [slots * rows][kvd] tensors; slot b's keys are rows b * rows + t.  Cross-
// attention: rows = seqlen and every slot attends all of them; self-attention:
// rows = the cache length and slot b attends min(pos[b] + 1, rows) keys.  CTA c
// loads rows [c * csz, c * csz + csz) of its kv head -- one [csz][64] TMA box for
// K and one for V -- into shared memory before any compute, so the whole chunk is
// in flight at once.
template <typename KV, bool kScores>
__global__ void __launch_bounds__(kThr) attn_kernel(const __grid_constant__ CUtensorMap tmK,
                                                    const __grid_constant__ CUtensorMap tmV, float *__restrict__ out,
                                                    const float *__restrict__ q, float *__restrict__ sc_out,
                                                    const uint32_t *__restrict__ pos, int rows, int nkv, int nh, int ns,
                                                    int csz, int *dev_err) {
    extern __shared__ uint8_t attn_smem[];
    KV *ks = reinterpret_cast<KV *>((reinterpret_cast<uintptr_t>(attn_smem) + 127) & ~uintptr_t(127));
    KV *vs = ks + (size_t)csz * kHd;
    __shared__ float qh[kHd];
    __shared__ float raw[kAttnMaxChunk];
    __shared__ float ew[kAttnMaxChunk];
    __shared__ float s8[8];
    __shared__ float red[8][kHd];
    __shared__ float part[8][2 + kHd];          // rank 0: the cluster's partials
    __shared__ float stats[2];                  // global (max, 1/sum), for the scores
    __shared__ __align__(8) uint64_t full;
    __shared__ int abort_flag;
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x;
    const int D = nh * kHd;
    const int kvh = h * nkv / nh;
    pdl_trigger();
    pdl_wait();                 // q, pos and the cache row at pos come from earlier kernels
    const int len = pos ? (pos[b] < (uint32_t)rows ? (int)pos[b] + 1 : rows) : rows;
    const int t0 = c * csz;
    int n = t0 < len ? min(csz, len - t0) : 0;
    if (ns > 1) asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
    if (tid == 0) {
        abort_flag = 0;
        mbar_init(&full, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0 && n > 0) {
        mbar_arrive_expect_tx(&full, (uint32_t)(2 * csz * kHd * sizeof(KV)));
        tma_load_2d(ks, &tmK, &full, kvh * kHd, b * rows + t0);
        tma_load_2d(vs, &tmV, &full, kvh * kHd, b * rows + t0);
    }
    if (tid < kHd) qh[tid] = q[(size_t)b * D + h * kHd + tid];
    bool landed = true;
    if (n > 0) landed = mbar_wait(&full, 0, &abort_flag, dev_err);
    __syncthreads();
    if (n > 0 && !__syncthreads_and(landed)) n = 0;     // a copy that never landed: contribute nothing
    scores_of(qh, ks, kHd, n, raw);
    __syncthreads();
    float lm = -INFINITY;
    for (int t = tid; t < n; t += kThr) lm = fmaxf(lm, raw[t]);
    const float mx = block_max(lm, s8);
    float ls = 0.f;
    for (int t = tid; t < n; t += kThr) {
        const float e = exp2f((raw[t] - mx) * kLog2e);
        ew[t] = e;
        ls += e;
    }
    const float ssum = block_sum(ls, s8);      // its barriers also publish ew[]
    const float o = pv_of(ew, vs, kHd, n, red);

    float *p0 = &part[0][0];
    if (ns > 1) {
        asm volatile("barrier.cluster.wait;" ::: "memory");
        p0 = cg::this_cluster().map_shared_rank(&part[0][0], 0);
    }
    if (tid < kHd) p0[c * (2 + kHd) + 2 + tid] = o;
    if (tid == 0) {
        p0[c * (2 + kHd)] = mx;
        p0[c * (2 + kHd) + 1] = ssum;
    }
    if (ns > 1) {
        asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
    } else {
        __syncthreads();
    }
    if (c == 0) {
        // log-sum-exp recombination (flash_cross_attn_reduce, decoder_ops.metal:416-457)
        float gm = -INFINITY;
        for (int r = 0; r < ns; ++r) gm = fmaxf(gm, part[r][0]);
        float gs = 0.f;
        for (int r = 0; r < ns; ++r)
            if (part[r][0] > -INFINITY) gs += part[r][1] * exp2f((part[r][0] - gm) * kLog2e);
        const float inv = 1.0f / gs;
        if (tid < kHd) {
            float acc = 0.f;
            for (int r = 0; r < ns; ++r)
                if (part[r][0] > -INFINITY) acc += part[r][2 + tid] * exp2f((part[r][0] - gm) * kLog2e);
            out[(size_t)b * D + h * kHd + tid] = acc * inv;
        }
        if constexpr (kScores) {
            if (tid < ns) {
                float *st = ns > 1 ? cg::this_cluster().map_shared_rank(stats, tid) : stats;
                st[0] = gm;
                st[1] = inv;
            }
        }
    }
    if constexpr (kScores) {
        if (ns > 1) asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
        else __syncthreads();
        const float gm = stats[0], inv = stats[1];
        float *sr = sc_out + ((size_t)b * nh + h) * rows + t0;
        for (int t = tid; t < n; t += kThr) sr[t] = exp2f((raw[t] - gm) * kLog2e) * inv;
    }
}

// ---------------------------------------------------------------- streamed attention
// The same (slot, head) clusters without the scores output, for any chunk size.
// CTA c walks its rows [c * csz, c * csz + n) in stages of kR rows (64 for f16
// K / V, 32 for f32: 16 KB of K and V per stage): a producer warp keeps a ring of
// `stages` TMA slots in flight ([kR][64] K and V boxes), and each of the 8
// consumer warps runs its own online softmax over its kR / 8 keys of every stage
// -- running max m_w, sum l_w and the partial output, rescaled by
// exp2((m_old - m_new) log2 e) when m_w grows -- with no block-wide barrier per
// stage.  A group of 8 lanes forms a key's score (4 keys per pass), each lane over
// 8 dims with packed f32x2 FMAs, and the same lane then accumulates p * v for its
// key over the same 8 dims (one 16-byte V load, no shuffle); the four groups'
// outputs are added after the stream.
// At the end the warps' (m, l, o) and then the cluster's CTAs are recombined by
// log-sum-exp, as flash_cross_attn_reduce does.
constexpr int kMaxStages = 8;
constexpr int kThrS = 288;                                 // 8 consumer warps + 1 producer warp

// The eight dims of a row that lane li of a key group handles (dim_of(li, i), i < 8):
// for f16 rows 8li .. 8li+7, for f32 rows 4li .. 4li+3 and 32+4li .. 32+4li+3, so
// that the 8 lanes of a group read 128 contiguous bytes per 16-byte load.
template <typename KV> MADI_DEV int dim_of(int li, int i);
template <> MADI_DEV int dim_of<__half>(int li, int i) { return 8 * li + i; }
template <> MADI_DEV int dim_of<float>(int li, int i) { return i < 4 ? 4 * li + i : 32 + 4 * li + (i - 4); }
// Those eight elements of a K or V row, as f32.
template <typename KV> MADI_DEV void ld8(const KV *r, int li, float (&f)[8]);
template <> MADI_DEV void ld8<__half>(const __half *r, int li, float (&f)[8]) {
    const uint4 u = *reinterpret_cast<const uint4 *>(r + 8 * li);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}
template <> MADI_DEV void ld8<float>(const float *r, int li, float (&f)[8]) {
    const float4 a = *reinterpret_cast<const float4 *>(r + 4 * li);
    const float4 b = *reinterpret_cast<const float4 *>(r + 32 + 4 * li);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
// This lane's part of q . k over its eight dims, in two interleaved f32 partial sums
// (packed f32x2 FMAs).
template <typename KV> MADI_DEV float dot8(const KV *kr, int li, const float (&qv)[8]) {
    float k[8];
    ld8<KV>(kr, li, k);
    float d0 = 0.f, d1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) fma2(d0, d1, qv[2 * i], qv[2 * i + 1], k[2 * i], k[2 * i + 1], d0, d1);
    return d0 + d1;
}

template <typename KV> struct StreamRows { static constexpr int kR = sizeof(KV) == 2 ? 64 : 32; };

// G heads per CTA (2 when every head has its own kv head and nh is even): the K / V
// boxes are G * 64 columns wide, so one TMA row request carries G heads' keys --
// the stream's rate is set by the number of box rows, not by their width -- and
// consumer warps 8/G * g .. 8/G * (g+1) - 1 serve head g.
template <typename KV, int G>
__global__ void __launch_bounds__(kThrS, 4) attn_stream_kernel(const __grid_constant__ CUtensorMap tmK,
                                                            const __grid_constant__ CUtensorMap tmV,
                                                            float *__restrict__ out, const float *__restrict__ q,
                                                            const uint32_t *__restrict__ pos, int rows, int nkv,
                                                            int nh, int ns, int csz, int stages, int *dev_err) {
    constexpr int kR = StreamRows<KV>::kR;
    constexpr int kW = kHd * G;                           // box width (elements)
    constexpr int kBox = kR * kW;                         // elements per K (or V) box
    constexpr int kWarpsPerHead = 8 / G;
    constexpr int kKeysPerWarp = kR / kWarpsPerHead;      // of each stage
    constexpr int kPasses = kKeysPerWarp / 4;             // 4 keys per pass
    extern __shared__ uint8_t attn_smem[];
    KV *ring = reinterpret_cast<KV *>((reinterpret_cast<uintptr_t>(attn_smem) + 127) & ~uintptr_t(127));
    __shared__ float qh[G][kHd];
    __shared__ float wm[8], wl[8];
    __shared__ float wo[8][kHd];
    __shared__ float part[8][G][2 + kHd];
    __shared__ __align__(8) uint64_t full[kMaxStages];
    __shared__ __align__(8) uint64_t empty[kMaxStages];
    __shared__ int abort_flag;
    const int c = blockIdx.x, hp = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int D = nh * kHd;
    const int kvh = hp * G * nkv / nh;                    // first kv head of the box (G > 1: nkv == nh)
    pdl_trigger();
    pdl_wait();                 // q, pos and the cache row at pos come from earlier kernels
    const int len = pos ? (pos[b] < (uint32_t)rows ? (int)pos[b] + 1 : rows) : rows;
    // Self-attention (pos given) splits the slot's actual keys 0..pos over the cluster,
    // not the cache's rows: every CTA streams its share of a short cache, none idles.
    const int cz = pos ? (len + ns - 1) / ns : csz;
    const int t0 = c * cz;
    const int n = t0 < len ? min(cz, len - t0) : 0;
    const int nsub = (n + kR - 1) / kR;
    if (ns > 1) asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
    if (tid == 0) {
        abort_flag = 0;
        for (int i = 0; i < stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 8);
        }
        fence_mbar_init();
    }
    if (tid < kHd * G) qh[tid / kHd][tid % kHd] = q[(size_t)b * D + hp * G * kHd + tid];
    __syncthreads();

    // consumer state: running max / sum of this warp and, per lane, its eight output
    // dims accumulated over the keys of the lane's group kq (summed over the four
    // groups after the stream)
    float m_w = -INFINITY, l_w = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (warp == 8) {
        // ------------------------------------------------ producer
        if (lane == 0) {
            const uint32_t tx = 2u * kBox * (uint32_t)sizeof(KV);
            int issued = 0;
            for (int j = 0; j < nsub; ++j) {
                const int s = j % stages;
                if (j >= stages && !mbar_wait(&empty[s], (uint32_t)(j / stages - 1) & 1u, &abort_flag, dev_err)) break;
                KV *ks = ring + (size_t)s * 2 * kBox;
                mbar_arrive_expect_tx(&full[s], tx);
                tma_load_2d(ks, &tmK, &full[s], kvh * kHd, b * rows + t0 + j * kR);
                tma_load_2d(ks + kBox, &tmV, &full[s], kvh * kHd, b * rows + t0 + j * kR);
                issued = j + 1;
            }
            // the copies issued last land before the CTA can exit
            for (int i2 = issued > stages ? issued - stages : 0; i2 < issued; ++i2) {
                const long long tw = clock64();
                while (!mbar_try_wait(&full[i2 % stages], (uint32_t)(i2 / stages) & 1u))
                    if (clock64() - tw > kWaitBudgetCycles) break;
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ consumers
        const int g = warp / kWarpsPerHead, wl_ = warp % kWarpsPerHead;
        const int li = lane & 7, kq = lane >> 3;          // 8 lanes per key, 4 keys per pass
        float qv[8];
#pragma unroll
        for (int i2 = 0; i2 < 8; ++i2) qv[i2] = qh[g][dim_of<KV>(li, i2)];
        const float rsq = rsqrtf((float)kHd);
        const int kb = wl_ * kKeysPerWarp;                // this warp's keys in each stage
        for (int j = 0; j < nsub; ++j) {
            const int s = j % stages;
            if (!warp_wait_all(&full[s], (uint32_t)(j / stages) & 1u, &abort_flag, dev_err)) {
                m_w = -INFINITY;                          // contribute nothing after a failed copy
                break;
            }
            const int rj = min(kR, n - j * kR);
            const KV *ks = ring + (size_t)s * 2 * kBox + g * kHd;
            const KV *vs = ks + kBox;
            float sc[kPasses];
            float mx = -INFINITY;
#pragma unroll
            for (int p = 0; p < kPasses; ++p) {
                const int k = kb + 4 * p + kq;
                float d = k < rj ? dot8<KV>(ks + (size_t)k * kW, li, qv) : 0.f;
                d += __shfl_xor_sync(0xffffffffu, d, 4);
                d += __shfl_xor_sync(0xffffffffu, d, 2);
                d += __shfl_xor_sync(0xffffffffu, d, 1);
                sc[p] = k < rj ? d * rsq : -INFINITY;
                mx = fmaxf(mx, sc[p]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            if (mx > -INFINITY) {                         // warp-uniform: this warp has keys here
                const float m_new = fmaxf(m_w, mx);
                const float alpha = exp2f((m_w - m_new) * kLog2e);
                m_w = m_new;
                l_w *= alpha;
#pragma unroll
                for (int i2 = 0; i2 < 8; i2 += 2) mul2(o[i2], o[i2 + 1], o[i2], o[i2 + 1], alpha, alpha);
#pragma unroll
                for (int p = 0; p < kPasses; ++p) {
                    const int k = kb + 4 * p + kq;          // this lane's key (the 8 lanes of kq agree on e)
                    const float e = exp2f((sc[p] - m_w) * kLog2e);     // 0 for a missing key
                    l_w += e;                                         // per key group; summed below
                    if (k < rj) {
                        float v[8];
                        ld8<KV>(vs + (size_t)k * kW, li, v);
#pragma unroll
                        for (int i2 = 0; i2 < 8; i2 += 2) fma2(o[i2], o[i2 + 1], e, e, v[i2], v[i2 + 1], o[i2], o[i2 + 1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // l_w and o hold the sums over one key group; the four groups are added
        l_w += __shfl_xor_sync(0xffffffffu, l_w, 8);
        l_w += __shfl_xor_sync(0xffffffffu, l_w, 16);
#pragma unroll
        for (int i2 = 0; i2 < 8; ++i2) {
            o[i2] += __shfl_xor_sync(0xffffffffu, o[i2], 8);
            o[i2] += __shfl_xor_sync(0xffffffffu, o[i2], 16);
        }
        if (kq == 0) {
#pragma unroll
            for (int i2 = 0; i2 < 8; ++i2) wo[warp][dim_of<KV>(li, i2)] = o[i2];
        }
        if (lane == 0) {
            wm[warp] = m_w;
            wl[warp] = l_w;
        }
    }
    __syncthreads();
    // this CTA's (m, l, o) per head: its warps' partials by log-sum-exp
    const int hg = tid / kHd, d = tid % kHd;              // threads 0 .. G*64-1: (head, dim)
    float cm = -INFINITY, cl = 0.f, co = 0.f;
    if (tid < kHd * G) {
#pragma unroll
        for (int w8 = 0; w8 < kWarpsPerHead; ++w8) cm = fmaxf(cm, wm[hg * kWarpsPerHead + w8]);
#pragma unroll
        for (int w8 = 0; w8 < kWarpsPerHead; ++w8) {
            const int w = hg * kWarpsPerHead + w8;
            if (wm[w] > -INFINITY) {
                const float f = exp2f((wm[w] - cm) * kLog2e);
                cl += wl[w] * f;
                co += wo[w][d] * f;
            }
        }
    }

    float *p0 = &part[0][0][0];
    if (ns > 1) {
        asm volatile("barrier.cluster.wait;" ::: "memory");
        p0 = cg::this_cluster().map_shared_rank(&part[0][0][0], 0);
    }
    if (tid < kHd * G) {
        float *pc = p0 + ((size_t)c * G + hg) * (2 + kHd);
        pc[2 + d] = co;
        if (d == 0) {
            pc[0] = cm;
            pc[1] = cl;
        }
    }
    if (ns > 1) {
        asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
    } else {
        __syncthreads();
    }
    if (c == 0 && tid < kHd * G) {
        float gm = -INFINITY;
        for (int r = 0; r < ns; ++r) gm = fmaxf(gm, part[r][hg][0]);
        float gs = 0.f, acc = 0.f;
        for (int r = 0; r < ns; ++r)
            if (part[r][hg][0] > -INFINITY) {
                const float f = exp2f((part[r][hg][0] - gm) * kLog2e);
                gs += part[r][hg][1] * f;
                acc += part[r][hg][2 + d] * f;
            }
        out[(size_t)b * D + (hp * G + hg) * kHd + d] = acc * (1.0f / gs);
    }
}

// Two-pass form with caller-owned partials part[head][nsplit][2 + 64] (m, s, o):
// pass 1, grid (nsplit, heads); raw scores to sc_raw[head][seqlen] when asked.
template <typename KV>
__global__ void __launch_bounds__(kThr) cross_attn_part_kernel(float *__restrict__ part, const float *__restrict__ q,
                                                               const KV *__restrict__ kc, const KV *__restrict__ vc,
                                                               float *__restrict__ sc_raw, int write_sc, int seqlen,
                                                               int kvd, int nkv, int nh, int nsplit) {
    __shared__ float qh[kHd];
    __shared__ float raw[kAttnMaxChunk];
    __shared__ float s8[8];
    __shared__ float red[8][kHd];
    const int c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    pdl_trigger();
    pdl_wait();
    const int kvh = h * nkv / nh;
    const int csz = (seqlen + nsplit - 1) / nsplit;
    const int t0 = c * csz;
    const int n = t0 < seqlen ? min(csz, seqlen - t0) : 0;
    float *my = part + ((size_t)h * nsplit + c) * (2 + kHd);
    if (n == 0) {                               // empty tail chunk
        if (tid == 0) { my[0] = -INFINITY; my[1] = 0.f; }
        if (tid < kHd) my[2 + tid] = 0.f;
        return;
    }
    const KV *kb = kc + (size_t)t0 * kvd + kvh * kHd;
    const KV *vb = vc + (size_t)t0 * kvd + kvh * kHd;
    if (tid < kHd) qh[tid] = q[h * kHd + tid];
    __syncthreads();
    scores_of(qh, kb, kvd, n, raw);
    __syncthreads();
    if (write_sc)
        for (int t = tid; t < n; t += kThr) sc_raw[(size_t)h * seqlen + t0 + t] = raw[t];
    float lm = -INFINITY;
    for (int t = tid; t < n; t += kThr) lm = fmaxf(lm, raw[t]);
    const float mx = block_max(lm, s8);
    float ls = 0.f;
    for (int t = tid; t < n; t += kThr) {
        const float e = exp2f((raw[t] - mx) * kLog2e);
        raw[t] = e;
        ls += e;
    }
    const float ssum = block_sum(ls, s8);
    const float o = pv_of(raw, vb, kvd, n, red);
    if (tid < kHd) my[2 + tid] = o;
    if (tid == 0) { my[0] = mx; my[1] = ssum; }
}

// pass 2, grid (heads): recombine and normalise the raw scores in place.
__global__ void __launch_bounds__(kThr) cross_attn_reduce_kernel(float *__restrict__ out, const float *__restrict__ part,
                                                                 int nsplit, float *__restrict__ sc, int seqlen,
                                                                 int write_sc) {
    const int h = blockIdx.x, tid = threadIdx.x;
    pdl_trigger();
    pdl_wait();
    const float *hp = part + (size_t)h * nsplit * (2 + kHd);
    float gm = -INFINITY;
    for (int c = 0; c < nsplit; ++c) gm = fmaxf(gm, hp[c * (2 + kHd)]);
    float gs = 0.f;
    for (int c = 0; c < nsplit; ++c) {
        const float m = hp[c * (2 + kHd)];
        if (m > -INFINITY) gs += hp[c * (2 + kHd) + 1] * exp2f((m - gm) * kLog2e);
    }
    const float inv = 1.0f / gs;
    if (tid < kHd) {
        float acc = 0.f;
        for (int c = 0; c < nsplit; ++c) {
            const float m = hp[c * (2 + kHd)];
            if (m > -INFINITY) acc += hp[c * (2 + kHd) + 2 + tid] * exp2f((m - gm) * kLog2e);
        }
        out[h * kHd + tid] = acc * inv;
    }
    if (write_sc) {
        float *sr = sc + (size_t)h * seqlen;
        for (int t = tid; t < seqlen; t += kThr) sr[t] = exp2f((sr[t] - gm) * kLog2e) * inv;
    }
}

// K / V as [slots * rows][kvd] with [csz][64] boxes (no swizzle: rows of 64
// elements, read conflict-free by half-warps).
bool attn_map(CUtensorMap *m, const void *base, bool f16, uint64_t total_rows, int kvd, int csz, int width = kHd) {
    PFN_encodeTiled enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)kvd, total_rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kvd * (f16 ? 2 : 4)};
    const cuuint32_t box[2] = {(cuuint32_t)width, (cuuint32_t)csz};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base),
               dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename KV, bool kScores>
cudaError_t launch_attn_t(const void *kc, const void *vc, float *out, const float *q, float *sc, const uint32_t *pos,
                          int slots, int rows, int kvd, int nkv, int nh, int *dev_err, cudaStream_t st) {
    const int ns = attn_cluster_size(rows);
    if (ns == 0) return cudaErrorInvalidValue;
    const int csz = (rows + ns - 1) / ns;
    const bool f16 = sizeof(KV) == 2;
    CUtensorMap tmK, tmV;
    if (!attn_map(&tmK, kc, f16, (uint64_t)slots * rows, kvd, csz) ||
        !attn_map(&tmV, vc, f16, (uint64_t)slots * rows, kvd, csz))
        return cudaErrorNotSupported;
    auto fn = attn_kernel<KV, kScores>;
    const size_t smem = 128 + 2 * (size_t)csz * kHd * sizeof(KV);
    static std::once_flag once;
    static cudaError_t once_status;
    if (cudaError_t e = run_once(once, once_status, [&] {
            return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)(128 + 2 * kAttnMaxChunk * kHd * sizeof(KV)));
        }))
        return e;
    return launch_k(fn, dim3(ns, nh, slots), kThr, smem, st, ns, tmK, tmV, out, q, sc, pos, rows, nkv, nh, ns, csz,
                    dev_err);
}

// One wave: the largest power-of-two ns (<= 8, >= 2 stages of rows per CTA) whose
// slots x heads x ns CTAs all fit at once, with the ring sized to the shared
// memory the resident CTAs leave (2..8 slots of 16 KB) and the fit checked against
// the occupancy the kernel really gets at that size; then another cluster size when
// it balances the SMs better (below).  MADI_ATTN_NS=1..8 in the environment forces
// the cluster size (for comparisons).
template <typename KV, int G>
cudaError_t launch_attn_stream_g(const void *kc, const void *vc, float *out, const float *q, const uint32_t *pos,
                                 int slots, int rows, int kvd, int nkv, int nh, int *dev_err, cudaStream_t st) {
    constexpr int kR = StreamRows<KV>::kR;
    constexpr size_t kSmemMax = 200 * 1024;
    const size_t stage_bytes = 2 * (size_t)kR * kHd * G * sizeof(KV);
    auto fn = attn_stream_kernel<KV, G>;
    static int occ[kMaxStages + 1] = {0};                 // resident CTAs per SM by ring depth
    static std::once_flag once;
    static cudaError_t once_status;
    if (cudaError_t e0 = run_once(once, once_status, [&] {
            cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)std::min(kSmemMax, 128 + kMaxStages * stage_bytes));
            if (e != cudaSuccess) return e;
            for (int sg = 2; sg <= kMaxStages; ++sg) {
                int nb = 0;
                if (128 + sg * stage_bytes <= kSmemMax) {
                    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, kThrS, 128 + sg * stage_bytes);
                    if (e != cudaSuccess) return e;
                }
                occ[sg] = nb;
            }
            return cudaSuccess;
        }))
        return e0;
    const int sms = num_sms();
    const long pairs = (long)slots * (nh / G);
    static const int forced_ns = [] {
        const char *e = getenv("MADI_ATTN_NS");
        const int v = e ? atoi(e) : 0;
        return v >= 1 && v <= 8 ? v : 0;
    }();
    auto ring_depth = [&](long per_sm) {
        const size_t budget = (size_t)(220 * 1024) / (size_t)per_sm;
        const size_t reserve = 12 * 1024;                // static shared memory and alignment
        int sg = budget > reserve ? (int)((budget - reserve) / stage_bytes) : 2;
        sg = sg < 2 ? 2 : (sg > kMaxStages ? kMaxStages : sg);
        while (sg > 2 && 128 + sg * stage_bytes > kSmemMax) --sg;
        return sg;
    };
    // Work on the busiest SM: resident CTAs x kR-row stages per CTA.
    auto busiest = [&](int cand, long per_sm) { return per_sm * (((rows + cand - 1) / cand + kR - 1) / kR); };
    int ns = 1, stages = 2;
    if (forced_ns) {
        ns = forced_ns;
        const long per_sm = (pairs * ns + sms - 1) / sms;
        stages = ring_depth(per_sm > 16 ? 16 : per_sm);
    } else {
        long best = -1;
        for (int cand = 8; cand >= 1; cand /= 2) {
            if (cand > 1 && (rows + cand - 1) / cand < 2 * kR) continue;
            const long per_sm = (pairs * cand + sms - 1) / sms;
            if (per_sm > 16) continue;
            const int sg = ring_depth(per_sm);
            if (occ[sg] >= per_sm || cand == 1) {
                ns = cand;
                stages = sg;
                best = busiest(cand, per_sm);
                break;
            }
        }
        // Cross-attention (every slot attends all `rows` keys): another cluster size (3,
        // 5 or 6 CTAs too) that also fits one wave with a ring of at least 3 stages
        // replaces it when it leaves less work on the busiest SM:
        // 8 slots x 10 head pairs give 320 CTAs at ns = 4, so 24 SMs hold a third CTA
        // and set the time; ns = 5 spreads 400 shorter CTAs.  Measured on a B200 (1500
        // f16 keys, min over 40 calls): 8 slots 22.4 -> 20.4 us, 2 slots 14.2 us at
        // ns = 6 (the same as 8), 15 slots unchanged at ns = 2.  Not taken: two-stage
        // rings (15 slots at ns = 3, 450 CTAs: 32.8 us against 30.6) and clusters of 7,
        // which pack into the GPCs worse than their per-SM occupancy says (2 and 4
        // slots: 20.3-20.5 us against 14.2-16.2 at 6 or 8).
        for (int cand = 8; cand >= 1 && best >= 0 && !pos; --cand) {
            if (cand == 7 || (cand > 1 && (rows + cand - 1) / cand < 2 * kR)) continue;
            const long per_sm = (pairs * cand + sms - 1) / sms;
            if (per_sm > 16) continue;
            const int sg = ring_depth(per_sm);
            if (sg < 3 || occ[sg] < per_sm) continue;
            const long c = busiest(cand, per_sm);
            if (c < best) {
                best = c;
                ns = cand;
                stages = sg;
            }
        }
    }
    const int csz = (rows + ns - 1) / ns;
    CUtensorMap tmK, tmV;
    const bool f16 = sizeof(KV) == 2;
    if (!attn_map(&tmK, kc, f16, (uint64_t)slots * rows, kvd, kR, kHd * G) ||
        !attn_map(&tmV, vc, f16, (uint64_t)slots * rows, kvd, kR, kHd * G))
        return cudaErrorNotSupported;
    return launch_k(fn, dim3(ns, nh / G, slots), kThrS, 128 + stages * stage_bytes, st, ns, tmK, tmV, out, q, pos,
                    rows, nkv, nh, ns, csz, stages, dev_err);
}

// Two heads per CTA when each head has its own kv head (Whisper's layout), else one.
// (Four heads per CTA measured slower: 31.5 us against 20.4 us at 8 slots x 1500 keys.)
template <typename KV>
cudaError_t launch_attn_stream(const void *kc, const void *vc, float *out, const float *q, const uint32_t *pos,
                               int slots, int rows, int kvd, int nkv, int nh, int *dev_err, cudaStream_t st) {
    if (nkv == nh && nh % 2 == 0)
        return launch_attn_stream_g<KV, 2>(kc, vc, out, q, pos, slots, rows, kvd, nkv, nh, dev_err, st);
    return launch_attn_stream_g<KV, 1>(kc, vc, out, q, pos, slots, rows, kvd, nkv, nh, dev_err, st);
}

}  // namespace

int attn_cluster_size(int seqlen) {
    int ns = 1;
    while (ns < 8 && (seqlen + ns - 1) / ns > 192) ns *= 2;
    return (seqlen + ns - 1) / ns <= kAttnMaxChunk ? ns : 0;
}

cudaError_t launch_cross_attn(float *out, const float *q, const void *kc, const void *vc, bool kv_f16, float *scores,
                              int slots, int seqlen, int kvd, int nkv, int nh, int *dev_err, cudaStream_t st) {
    if (kv_f16)
        return scores ? launch_attn_t<__half, true>(kc, vc, out, q, scores, nullptr, slots, seqlen, kvd, nkv, nh, dev_err, st)
                      : launch_attn_stream<__half>(kc, vc, out, q, nullptr, slots, seqlen, kvd, nkv, nh, dev_err, st);
    return scores ? launch_attn_t<float, true>(kc, vc, out, q, scores, nullptr, slots, seqlen, kvd, nkv, nh, dev_err, st)
                  : launch_attn_stream<float>(kc, vc, out, q, nullptr, slots, seqlen, kvd, nkv, nh, dev_err, st);
}

cudaError_t launch_cross_attn_part(float *part, const float *q, const void *kc, const void *vc, bool kv_f16,
                                   float *sc_raw, int write_sc, int seqlen, int kvd, int nkv, int nh, int nsplit,
                                   cudaStream_t st) {
    const dim3 grid(nsplit, nh);
    if (kv_f16)
        return launch_k(cross_attn_part_kernel<__half>, grid, kThr, 0, st, 1, part, q, static_cast<const __half *>(kc),
                        static_cast<const __half *>(vc), sc_raw, write_sc, seqlen, kvd, nkv, nh, nsplit);
    return launch_k(cross_attn_part_kernel<float>, grid, kThr, 0, st, 1, part, q, static_cast<const float *>(kc),
                    static_cast<const float *>(vc), sc_raw, write_sc, seqlen, kvd, nkv, nh, nsplit);
}

cudaError_t launch_cross_attn_reduce(float *out, const float *part, int nsplit, float *sc, int seqlen, int write_sc,
                                     int nh, cudaStream_t st) {
    return launch_k(cross_attn_reduce_kernel, nh, kThr, 0, st, 1, out, part, nsplit, sc, seqlen, write_sc);
}

// ---------------------------------------------------------------- fixed-scratch split form
// Partials [heads][nsplit][2 + 64] of madi_cross_attn_split_static.  Every GPU that
// loads the library holds this array (540 672 bytes) until the process exits; host
// code only ever sees a stand-in for it, so kernels get the device address that
// cudaGetSymbolAddress returns for the current device.  The split pass writes every
// (head, split) entry it covers before the reduce pass reads it, so nothing needs
// clearing between calls.
static __device__ __align__(256) float g_split_part[kSplitStaticMax * (2 + kHd)];

// The array's address is looked up once per device and context: the entry for a
// device is refreshed when the current context is another one (the context was
// destroyed and created again, e.g. after cudaDeviceReset).
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_split_mu;
struct SplitAddr {
    CUcontext ctx = nullptr;
    float *addr = nullptr;
} g_split_addr[kMaxDevices];

CUcontext current_context() {
    typedef CUresult (*PFN_ctx)(CUcontext *);
    static PFN_ctx fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_ctx>(ptr);
    });
    CUcontext c = nullptr;
    if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}
}  // namespace

void forget_split_static_addresses() {
    std::lock_guard<std::mutex> lk(g_split_mu);
    for (auto &a : g_split_addr) a = SplitAddr();
}

cudaError_t launch_cross_attn_split_static(float *out, const float *q, const void *kc, const void *vc, float *sc,
                                           int seqlen, int kvd, int nkv, int nh, int nsplit, int device,
                                           cudaStream_t st) {
    if ((long)nh * nsplit > kSplitStaticMax) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != device || dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    float *part = nullptr;
    {
        // the first call on this device (and context) makes the context current
        // through cudaGetSymbolAddress; the context is read after it
        std::lock_guard<std::mutex> lk(g_split_mu);
        SplitAddr &a = g_split_addr[dev];
        CUcontext ctx = current_context();
        if (!a.addr || !ctx || ctx != a.ctx) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_split_part);
            if (e != cudaSuccess) return e;
            a.addr = static_cast<float *>(p);
            a.ctx = current_context();
        }
        part = a.addr;
    }
    e = launch_cross_attn_part(part, q, kc, vc, true, sc, sc != nullptr, seqlen, kvd, nkv, nh, nsplit, st);
    if (e != cudaSuccess) return e;
    return launch_cross_attn_reduce(out, part, nsplit, sc, seqlen, sc != nullptr, nh, st);
}

cudaError_t launch_self_attn(float *out, const float *q, const void *kc, const void *vc, bool kv_f16,
                             const uint32_t *pos, int slots, int kvd, int nkv, int nh, int max_tok, int *dev_err,
                             cudaStream_t st) {
    return kv_f16 ? launch_attn_stream<__half>(kc, vc, out, q, pos, slots, max_tok, kvd, nkv, nh, dev_err, st)
                  : launch_attn_stream<float>(kc, vc, out, q, pos, slots, max_tok, kvd, nkv, nh, dev_err, st);
}

}  // namespace madi
