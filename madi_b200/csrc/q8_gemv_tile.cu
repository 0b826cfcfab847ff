// q8_gemv_tile.cu -- variant (b): the decode Q8_0 GEMV / skinny GEMM (M <= 8) for
// every shape with K % 256 == 0 (all Whisper decoder projections and the vocab
// head).  q8_gemv.cu keeps the shapes this kernel does not take.
//
// Arithmetic (graph_helpers.metal:320-567, f32 throughout), as in q8_gemv.cu:
// int8 weights become f16 exactly, each 32-block's partial sum is scaled by its
// f16 scale in f32, f32 activations are split into f16 hi + lo (hi = f16(x),
// lo = f16(x - hi)), and mma.sync m16n8k16 accumulates in f32.
//
// Data movement:
//   * a unit of work is one 16-row tile of W over a K-slice: all of K, or 1/cs of
//     it when a thread-block cluster of cs CTAs splits K.  A producer warp moves a
//     unit into one shared-memory stage with tiled TMA: KS/256 boxes of
//     [16 rows][2][128 B] under the 128-byte swizzle (the weights viewed as
//     [N][K/128][128]) and one [16][KS/32] box of scales; rows past N arrive
//     zero-filled.  The producer runs ahead of griddepcontrol.wait: weights do not
//     depend on the previous kernel, so under programmatic dependent launch they
//     stream while that kernel drains;
//   * 8 consumer warps share every unit: warp w takes the 32-blocks kb = w, w + 8,
//     ... of the slice.  With kb mod 8 fixed per warp a lane's fragment address
//     inside a box is a constant, and the swizzle puts the four rows a half-warp
//     reads in four different bank groups (conflict-free 8-byte loads).  The x
//     slice is staged once per CTA in fragment order;
//   * the 8 partial [16 x 8] results meet in shared memory (double-buffered) and
//     warp (unit mod 8) adds them in warp order, then runs the epilogue.  Under a
//     K split each cluster owns exactly one unit: every rank pushes its CTA sum
//     into rank 0's shared memory, where the sums are added in rank order.  All
//     sums have a fixed order, so results are run-to-run identical;
//   * CTAs are small (9 warps, <= 112 registers, shared memory sized for two per
//     SM where possible), which also leaves room for the next kernel's CTAs to
//     start and prefetch beside them.  With more units than CTA slots the grid is
//     persistent: cluster c walks units c, c + clusters, ...
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace cg = cooperative_groups;

namespace madi {
namespace {

constexpr int kConsumers = 8;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kTileRows = 16;
constexpr int kMaxStages = 8;
constexpr int kMaxCs = 4;
constexpr int kBoxBytes = kTileRows * 256;                  // one [16][2][128 B] weight box
constexpr int kMaxM = 16;                                   // token rows: 1 or 2 groups of 8 (the MMA's n)
constexpr size_t kRedBytes = 2 * kConsumers * 32 * 16;      // per token group: 2 units x 8 warps x 32 lanes x float4
constexpr size_t kXredBytes = kMaxCs * 32 * 16;             // per token group and unit: per-rank CTA sums, on rank 0
constexpr int kSplitUnits = 2;                              // units per CTA of a K-split plan, at most
constexpr size_t kSmemCap = 227 * 1024;                     // opt-in maximum per CTA
constexpr size_t kSmemHalf = 112 * 1024;                    // two CTAs per SM (228 KB less reserves)

struct __align__(8) TileBars {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    int abort;
};

struct TilePlan {
    int cs;          // CTAs per cluster = K slices per unit (1, 2, 4)
    int kslice;      // K per CTA, a multiple of 256
    int stages;      // ring depth
    int clusters;    // clusters in the grid (== units when cs > 1)
};

// One stage: the KS/256 weight boxes back to back (16 x KS bytes), then the
// 16 x KS/32 scales; rounded to 1 KB so each stage starts on the swizzle period.
__host__ __device__ constexpr size_t stage_bytes(int KS) {
    return ((size_t)kTileRows * KS + (size_t)kTileRows * (KS / 32) * 2 + 1023) & ~size_t(1023);
}
__host__ __device__ constexpr size_t x_bytes(int M, int KS, bool x_f32) { return (size_t)M * KS * (x_f32 ? 4 : 2); }
__host__ __device__ constexpr int groups(int M) { return (M + 7) / 8; }
__host__ __device__ constexpr size_t fixed_bytes(int M, int KS, bool x_f32) {
    return 1024 + x_bytes(M, KS, x_f32) + (size_t)groups(M) * (kRedBytes + kSplitUnits * kXredBytes) +
           sizeof(TileBars);
}
size_t plan_smem(int M, const TilePlan &pl, bool x_f32) {
    return fixed_bytes(M, pl.kslice, x_f32) + (size_t)pl.stages * stage_bytes(pl.kslice);
}

// Launch plan.  Split K over a cluster when the units then still fit one wave at
// two CTAs per SM (more CTAs streaming, fewer blocks per warp); otherwise one CTA
// per unit, persistent when units outnumber the CTA slots.  Two CTAs per SM when
// shared memory allows, else one.  Last resort, a K split over more than a wave.
bool make_plan(int M, int N, int K, bool x_f32, int num_sms, TilePlan *pl, int *grid) {
    if (M < 1 || M > kMaxM || N < 1 || K < 256 || K % 256 != 0) return false;
    const int tiles = (N + kTileRows - 1) / kTileRows;
    for (int cs = kMaxCs; cs >= 2; cs /= 2) {
        if (K % (256 * cs) != 0 || (long)tiles * cs > 2L * num_sms) continue;
        const TilePlan c{cs, K / cs, 1, tiles};
        if (c.kslice / 32 > 256 || plan_smem(M, c, x_f32) > kSmemHalf) continue;
        *pl = c;
        *grid = tiles * cs;
        return true;
    }
    // K split with two units per CTA (the second unit's weights load while the first
    // is computed) when one unit per CTA needs more than a wave and the wider x slice
    // of a one-unit split does not fit two CTAs per SM (16 token rows, K = 5120).
    for (int cs = kMaxCs; cs >= 2; cs /= 2) {
        const int clusters = (tiles + kSplitUnits - 1) / kSplitUnits;
        if (K % (256 * cs) != 0 || (long)clusters * cs > 2L * num_sms) continue;
        const TilePlan c{cs, K / cs, kSplitUnits, clusters};
        if (c.kslice / 32 > 256 || plan_smem(M, c, x_f32) > kSmemHalf) continue;
        *pl = c;
        *grid = clusters * cs;
        return true;
    }
    for (int per_sm = 2; per_sm >= 1 && K / 32 <= 256; --per_sm) {   // one scale box per unit
        const size_t budget = per_sm == 2 ? kSmemHalf : kSmemCap;
        const int clusters = tiles < per_sm * num_sms ? tiles : per_sm * num_sms;
        const int units = (tiles + clusters - 1) / clusters;   // per CTA
        const size_t fixed = fixed_bytes(M, K, x_f32);
        if (fixed + stage_bytes(K) > budget) continue;
        int stages = (int)((budget - fixed) / stage_bytes(K));
        if (stages > kMaxStages) stages = kMaxStages;
        if (stages > units) stages = units;
        if (units > 1 && stages < 2) continue;          // a lone stage cannot overlap load and compute
        *pl = TilePlan{1, K, stages, clusters};
        *grid = clusters;
        return true;
    }
    // Neither fits (an f32 x slice of a long K, e.g. 8 or 16 x 5120): split K even
    // though the clusters then take more than one wave, at two CTAs per SM if the
    // slice fits, else one.
    for (const size_t budget : {kSmemHalf, kSmemCap}) {
        for (int cs = kMaxCs; cs >= 2; cs /= 2) {
            if (K % (256 * cs) != 0) continue;
            const TilePlan c{cs, K / cs, 1, tiles};
            if (c.kslice / 32 > 256 || plan_smem(M, c, x_f32) > budget) continue;
            *pl = c;
            *grid = tiles * cs;
            return true;
        }
    }
    return false;
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

// Writes one unit's outputs: v = (row g8, tokens tok0 + 2t, tok0 + 2t+1), (row g8 + 8, same).
template <typename YT, int EPI, bool kQKV>
MADI_DEV void store_unit(const GemvArgs &p, int tile, int g8, int t, int tok0, const float4 &v4) {
    const float v[4] = {v4.x, v4.y, v4.z, v4.w};
    const int row0 = tile * kTileRows + g8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = (i < 2) ? row0 : row0 + 8;
        const int tok = tok0 + 2 * t + (i & 1);
        if (row >= p.N || tok >= p.M) continue;
        float y = v[i];
        if constexpr (kQKV) {
            // gemv_q8_qkv (graph_helpers.metal:527-567): q + qb -> q_out, k -> kc[pos],
            // v + vb -> vc[pos]
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
            if constexpr (EPI == kEpiBiasRes) y = s_to_f32(reinterpret_cast<const YT *>(p.residual)[o]) + y + b;
            reinterpret_cast<YT *>(p.y)[o] = s_from_f32<YT>(y);
        }
    }
}

// One quad column (4 consecutive k) of all M token rows of x: load = true fetches
// it into v, load = false converts v and stores it in fragment order.  kR16: f32 x
// rounded to f16 when staged (stored as f16 x is).
template <typename XT, int kRows, bool kR16>
MADI_DEV void stage_x_quad(const GemvArgs &p, uint8_t *xs, const XT *xrow, int kq, bool have,
                           typename std::conditional<sizeof(XT) == 4, float4, uint2>::type (&v)[kRows], bool load) {
    constexpr bool kSplit = sizeof(XT) == 4;
    const int M = p.M, K = p.K;
    const int kl = kq << 2;
    if (!have) return;
    if (load) {
#pragma unroll
        for (int m = 0; m < kRows; ++m)
            if (m < M) {
                if constexpr (kSplit) v[m] = __ldcg(reinterpret_cast<const float4 *>(xrow + (size_t)m * K + kl));
                else v[m] = __ldcg(reinterpret_cast<const uint2 *>(xrow + (size_t)m * K + kl));
            }
        return;
    }
    const int slot0 = ((kl >> 5) * 2 + ((kl & 7) >> 2)) * M * 4 + ((kl & 31) >> 3);
#pragma unroll
    for (int m = 0; m < kRows; ++m)
        if (m < M) {
            if constexpr (kSplit && kR16) {
                const float4 f = v[m];
                reinterpret_cast<uint2 *>(xs)[slot0 + m * 4] =
                    make_uint2(h2_as_u32(__floats2half2_rn(f.x, f.y)), h2_as_u32(__floats2half2_rn(f.z, f.w)));
            } else if constexpr (kSplit) {
                const float4 f = v[m];
                const __half2 h01 = __floats2half2_rn(f.x, f.y);
                const __half2 h23 = __floats2half2_rn(f.z, f.w);
                const __half2 l01 = __floats2half2_rn(f.x - __low2float(h01), f.y - __high2float(h01));
                const __half2 l23 = __floats2half2_rn(f.z - __low2float(h23), f.w - __high2float(h23));
                reinterpret_cast<uint4 *>(xs)[slot0 + m * 4] =
                    make_uint4(h2_as_u32(h01), h2_as_u32(h23), h2_as_u32(l01), h2_as_u32(l23));
            } else {
                reinterpret_cast<uint2 *>(xs)[slot0 + m * 4] = v[m];
            }
        }
}

// Stage the x slice [M][kb0*32, kb0*32 + KS) once in fragment order: slot
// (lkb, s, m, t) holds x[m][(kb0 + lkb)*32 + 8t + 4s + 0..3] as f16 hi (and, for
// f32 x, f16 lo) pairs.  Thread `tid` of `nthr` owns the quads kq = tid, tid +
// nthr, ... and fetches a quad of all M token rows at once; two quads' loads are
// in flight before either is converted, so a slice of up to 2 * nthr quads costs
// one L2 round trip.  x may have been written by the kernel this one overlaps
// under programmatic dependent launch, so it is read on the coherent L2 path
// (ld.global.cg), never through the non-coherent one.
template <typename XT, int kG, bool kR16>
MADI_DEV void stage_x(const GemvArgs &p, uint8_t *xs, int kb0, int KS, int tid, int nthr) {
    using V = typename std::conditional<sizeof(XT) == 4, float4, uint2>::type;
    const int qrow = KS >> 2;
    const XT *xrow = reinterpret_cast<const XT *>(p.x) + (size_t)kb0 * 32;
    if constexpr (kG == 1) {
        for (int kq = tid; kq < qrow; kq += 2 * nthr) {
            V a[8], b[8];
            const bool hb = kq + nthr < qrow;
            stage_x_quad<XT, 8, kR16>(p, xs, xrow, kq, true, a, true);
            stage_x_quad<XT, 8, kR16>(p, xs, xrow, kq + nthr, hb, b, true);
            stage_x_quad<XT, 8, kR16>(p, xs, xrow, kq, true, a, false);
            stage_x_quad<XT, 8, kR16>(p, xs, xrow, kq + nthr, hb, b, false);
        }
    } else if constexpr (sizeof(XT) == 2) {
        // 16 rows of f16 x: two quads' loads (32 x 8 bytes) in flight before either is
        // stored, as for 8 rows -- a K = 1280 slice then costs one L2 round trip
        for (int kq = tid; kq < qrow; kq += 2 * nthr) {
            V a[16], b[16];
            const bool hb = kq + nthr < qrow;
            stage_x_quad<XT, 16, kR16>(p, xs, xrow, kq, true, a, true);
            stage_x_quad<XT, 16, kR16>(p, xs, xrow, kq + nthr, hb, b, true);
            stage_x_quad<XT, 16, kR16>(p, xs, xrow, kq, true, a, false);
            stage_x_quad<XT, 16, kR16>(p, xs, xrow, kq + nthr, hb, b, false);
        }
    } else {
        for (int kq = tid; kq < qrow; kq += nthr) {      // 16 rows of f32: one quad's loads at a time
            V a[16];
            stage_x_quad<XT, 16, kR16>(p, xs, xrow, kq, true, a, true);
            stage_x_quad<XT, 16, kR16>(p, xs, xrow, kq, true, a, false);
        }
    }
}

// kG: token groups of 8 (1 for M <= 8, 2 for 9..16); each weight fragment feeds
// one m16n8k16 MMA per group.
// kR16: f32 x rounded to f16 when staged, then the f16 path (one MMA per group).
template <typename XT, typename YT, int EPI, bool kQKV, int kG, bool kR16>
__global__ void __launch_bounds__(kThreads, 2)
    q8_gemv_tile_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tms,
                        const GemvArgs p, const TilePlan plan, int *dev_err) {
    constexpr bool kSplit = sizeof(XT) == 4 && !kR16;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int M = p.M, N = p.N;
    const int cs = plan.cs, KS = plan.kslice, stages = plan.stages, clusters = plan.clusters;
    const int nkbs = KS >> 5;                                   // 32-blocks in this CTA's slice
    const int rank = (int)(blockIdx.x % (unsigned)cs);          // cluster rank (clusters run along x)
    const int cl = (int)(blockIdx.x / (unsigned)cs);
    const int kb0 = rank * nkbs;                                // first block of the slice
    const size_t sb = stage_bytes(KS);
    uint8_t *ring = smem;
    uint8_t *xs = smem + (size_t)stages * sb;
    float4 *red = reinterpret_cast<float4 *>(xs + x_bytes(M, KS, kSplit));
    float4 *xred = red + 2 * kConsumers * 32 * kG;
    TileBars *bars = reinterpret_cast<TileBars *>(reinterpret_cast<uint8_t *>(xred) + kG * kSplitUnits * kXredBytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g8 = lane >> 2, t = lane & 3;
    const int tiles = (N + kTileRows - 1) / kTileRows;
    volatile int *abort_flag = &bars->abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], kConsumers);
        }
        bars->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    // Under a K split, rank 0's shared memory receives the other ranks' sums: the
    // arrive here and the wait before the first remote store make sure every CTA
    // of the cluster is running by then.
    if (cs > 1) asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");

    // Reducer lanes of a split unit: `mine` holds the CTA sums of unit `mine_unit`.  A
    // CTA's units are reduced by different warps (unit n by warp n), so a thread holds
    // the sums of one unit at most.
    bool have = false;
    float4 mine[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) mine[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    int mine_tile = 0, mine_unit = 0;

    if (warp == 0) {
        // ------------------------------------------------ producer: one stage = one unit
        if (lane == 0) {
            tma_prefetch_desc(&tmq);
            tma_prefetch_desc(&tms);
            const uint32_t tx = (uint32_t)(KS / 256) * kBoxBytes + (uint32_t)kTileRows * nkbs * 2;
            const int c1 = kb0 >> 2;                            // 128-byte chunk where the slice starts
            int s = 0;
            uint32_t ph = 0;
            uint32_t issued = 0, last_ph[kMaxStages];
            for (int tile = cl; tile < tiles; tile += clusters) {
                if (!mbar_wait(&bars->empty[s], ph ^ 1, abort_flag, dev_err)) break;
                const int r0 = tile * kTileRows;
                uint8_t *st = ring + (size_t)s * sb;
                mbar_arrive_expect_tx(&bars->full[s], tx);
                for (int o = 0; o < KS / 256; ++o)
                    tma_load_3d(st + o * kBoxBytes, &tmq, &bars->full[s], 0, c1 + 2 * o, r0);
                tma_load_2d(st + (size_t)kTileRows * KS, &tms, &bars->full[s], kb0, r0);
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
        __syncwarp();
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    } else {
        // ------------------------------------------------ consumers
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        asm volatile("griddepcontrol.wait;" ::: "memory");
        stage_x<XT, kG, kR16>(p, xs, kb0, KS, (int)threadIdx.x - 32, kConsumers * 32);
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");   // consumers only

        const int cw = warp - 1;
        bool gval[kG];
#pragma unroll
        for (int g = 0; g < kG; ++g) gval[g] = g8 + 8 * g < M;
        const int nki = nkbs >> 3;                          // 32-blocks per warp per unit
        const uint32_t off0 = frag_offset(g8, cw, t), off1 = frag_offset(g8 + 8, cw, t);
        const int xstep = 16 * M * 4;                       // x slots per i (8 blocks x 2 halves x M x 4)
        const int xbase = (cw * 2 * M + g8) * 4 + t;        // slot of (lkb = cw, s = 0, m = g8, t)
        bool alive = true;
        // Every consumer warp runs every unit of the CTA, so the named barrier below
        // is met by all 256 consumer threads each time, also after a bounded wait
        // gave up; each warp waited for a stage's previous round itself, so the
        // parity waits are unambiguous.
        int s = 0;                                          // stage and parity of unit n, division-free
        uint32_t ph = 0;
        for (int n = 0, tile = cl; tile < tiles; ++n, tile += clusters, s = (s + 1 == stages) ? 0 : s + 1,
                 ph ^= (s == 0) ? 1u : 0u) {
            if (alive) alive = warp_wait_all(&bars->full[s], ph, abort_flag, dev_err);
            float acc[kG][4];
#pragma unroll
            for (int g = 0; g < kG; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
            if (alive) {
                const uint8_t *st = ring + (size_t)s * sb;
                const __half *sc = reinterpret_cast<const __half *>(st + (size_t)kTileRows * KS);
                const __half *s0p = sc + g8 * nkbs + cw, *s1p = s0p + 8 * nkbs;
#pragma unroll 4
                for (int i = 0; i < nki; ++i) {
                    const uint2 wa = *reinterpret_cast<const uint2 *>(st + off0 + i * kBoxBytes);
                    const uint2 wb = *reinterpret_cast<const uint2 *>(st + off1 + i * kBoxBytes);
                    // the block's products (both k16 halves; for f32 x, hi and lo) meet in
                    // one f32 accumulator, then take the block scale
                    float bs[kG][4];
#pragma unroll
                    for (int g = 0; g < kG; ++g) bs[g][0] = bs[g][1] = bs[g][2] = bs[g][3] = 0.f;
#pragma unroll
                    for (int sp = 0; sp < 2; ++sp) {
                        __half2 a_lo0, a_hi0, a_lo1, a_hi1;
                        q8_to_half2x2(sp == 0 ? wa.x : wa.y, a_lo0, a_hi0);
                        q8_to_half2x2(sp == 0 ? wb.x : wb.y, a_lo1, a_hi1);
                        const uint32_t a[4] = {h2_as_u32(a_lo0), h2_as_u32(a_lo1), h2_as_u32(a_hi0), h2_as_u32(a_hi1)};
                        const int slot = xbase + i * xstep + sp * M * 4;
#pragma unroll
                        for (int g = 0; g < kG; ++g) {              // tokens 8g .. 8g+7: slots 32 further
                            if constexpr (kSplit) {
                                const uint4 xv = gval[g] ? reinterpret_cast<const uint4 *>(xs)[slot + 32 * g]
                                                         : make_uint4(0u, 0u, 0u, 0u);
                                mma16816(bs[g], a, xv.x, xv.y);
                                mma16816(bs[g], a, xv.z, xv.w);
                            } else {
                                const uint2 xv = gval[g] ? reinterpret_cast<const uint2 *>(xs)[slot + 32 * g]
                                                         : make_uint2(0u, 0u);
                                mma16816(bs[g], a, xv.x, xv.y);
                            }
                        }
                    }
                    const float f0 = __half2float(s0p[8 * i]);
                    const float f1 = __half2float(s1p[8 * i]);
#pragma unroll
                    for (int g = 0; g < kG; ++g) {
                        acc[g][0] = fmaf(bs[g][0], f0, acc[g][0]);
                        acc[g][1] = fmaf(bs[g][1], f0, acc[g][1]);
                        acc[g][2] = fmaf(bs[g][2], f1, acc[g][2]);
                        acc[g][3] = fmaf(bs[g][3], f1, acc[g][3]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->empty[s]);   // stage consumed: the producer may refill it
            float4 *rb = red + (size_t)(n & 1) * kConsumers * 32 * kG;
#pragma unroll
            for (int g = 0; g < kG; ++g)
                rb[(cw * kG + g) * 32 + lane] = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
            asm volatile("bar.sync 2, %0;" ::"r"(kConsumers * 32) : "memory");
            // The reducer of unit n reads buffer n & 1 before it reaches the barrier of
            // unit n + 1, and unit n + 2 rewrites that buffer only after that barrier.
            if (cw != (n & (kConsumers - 1))) continue;
#pragma unroll
            for (int g = 0; g < kG; ++g) {
                float4 v = rb[g * 32 + lane];
#pragma unroll
                for (int w = 1; w < kConsumers; ++w) {
                    const float4 q = rb[(w * kG + g) * 32 + lane];
                    v.x += q.x; v.y += q.y; v.z += q.z; v.w += q.w;
                }
                if (cs > 1) mine[g] = v;
                else if (alive) store_unit<YT, EPI, kQKV>(p, tile, g8, t, 8 * g, v);
            }
            if (cs > 1) {
                mine_tile = tile;
                mine_unit = n;
                have = alive;
            }
        }
    }

    if (cs > 1) {
        // At most kSplitUnits units per cluster: ranks push their CTA sums into rank 0
        // (a slot per unit and rank), which adds them in rank order.  Every thread of
        // every CTA takes part in both barriers.
        cg::cluster_group cluster = cg::this_cluster();
        asm volatile("barrier.cluster.wait;" ::: "memory");
        if (have) {
#pragma unroll
            for (int g = 0; g < kG; ++g)
                cluster.map_shared_rank(xred, 0)[((mine_unit * cs + rank) * kG + g) * 32 + lane] = mine[g];
        }
        asm volatile("barrier.cluster.arrive.release;" ::: "memory");
        asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
        if (rank == 0 && have) {
#pragma unroll
            for (int g = 0; g < kG; ++g) {
                float4 v = xred[(mine_unit * cs * kG + g) * 32 + lane];
                for (int r = 1; r < cs; ++r) {
                    const float4 q = xred[((mine_unit * cs + r) * kG + g) * 32 + lane];
                    v.x += q.x; v.y += q.y; v.z += q.z; v.w += q.w;
                }
                store_unit<YT, EPI, kQKV>(p, mine_tile, g8, t, 8 * g, v);
            }
        }
    }
}

// Weights as a 3-D tensor [N][K/128][128] (bytes) read in [16][2][128] boxes with
// the 128-byte swizzle; scales as a 2-D tensor [N][K/32] (u16) read in
// [16][KS/32] boxes.  Out-of-range rows are zero-filled.
bool make_tile_maps(const GemvArgs &a, int KS, CUtensorMap *tmq, CUtensorMap *tms) {
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
    const cuuint32_t sbox[2] = {(cuuint32_t)KS / 32, kTileRows};
    return enc(tms, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<__half *>(a.scales), sd, sstr, sbox, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename XT, typename YT, int EPI, bool kQKV, int kG, bool kR16>
cudaError_t launch_tile_g(const GemvArgs &a, const CUtensorMap &tmq, const CUtensorMap &tms, const TilePlan &pl,
                          int grid, int *dev_err, cudaStream_t st, bool pdl) {
    auto fn = q8_gemv_tile_kernel<XT, YT, EPI, kQKV, kG, kR16>;
    static std::once_flag once;
    static cudaError_t once_status;
    if (cudaError_t e = run_once(once, once_status, [&] {
            return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap);
        }))
        return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = plan_smem(a.M, pl, sizeof(XT) == 4 && !kR16);
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    int na = 0;
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    ++na;
    if (pl.cs > 1) {
        attrs[na].id = cudaLaunchAttributeClusterDimension;
        attrs[na].val.clusterDim.x = pl.cs;
        attrs[na].val.clusterDim.y = 1;
        attrs[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, fn, tmq, tms, a, pl, dev_err);
}

template <typename XT, typename YT, int EPI, bool kQKV, bool kR16 = false>
cudaError_t launch_tile_one(const GemvArgs &a, const CUtensorMap &tmq, const CUtensorMap &tms, const TilePlan &pl,
                            int grid, int *dev_err, cudaStream_t st, bool pdl) {
    return a.M > 8 ? launch_tile_g<XT, YT, EPI, kQKV, 2, kR16>(a, tmq, tms, pl, grid, dev_err, st, pdl)
                   : launch_tile_g<XT, YT, EPI, kQKV, 1, kR16>(a, tmq, tms, pl, grid, dev_err, st, pdl);
}

}  // namespace

bool gemv_tile_ok(int M, int N, int K, bool x_f32, int num_sms) {
    TilePlan pl;
    int grid;
    return make_plan(M, N, K, x_f32, num_sms, &pl, &grid);
}

cudaError_t launch_gemv_tile(const GemvArgs &a, bool x_f32, bool y_f32, int epi, bool qkv, int num_sms, int *dev_err,
                             cudaStream_t st, bool pdl, bool x_r16) {
    TilePlan pl;
    int grid;
    if (x_r16 && !x_f32) return cudaErrorInvalidValue;
    if (!make_plan(a.M, a.N, a.K, x_f32 && !x_r16, num_sms, &pl, &grid)) return cudaErrorInvalidValue;
    CUtensorMap tmq, tms;
    if (!make_tile_maps(a, pl.kslice, &tmq, &tms)) return cudaErrorNotSupported;
    if (qkv) {
        if (!x_f32) return launch_tile_one<__half, float, kEpiNone, true>(a, tmq, tms, pl, grid, dev_err, st, pdl);
        return x_r16 ? launch_tile_one<float, float, kEpiNone, true, true>(a, tmq, tms, pl, grid, dev_err, st, pdl)
                     : launch_tile_one<float, float, kEpiNone, true>(a, tmq, tms, pl, grid, dev_err, st, pdl);
    }
#define MADI_TILE_CASE(XT, YT)                                                                                   \
    switch (epi) {                                                                                               \
        case kEpiNone: return launch_tile_one<XT, YT, kEpiNone, false>(a, tmq, tms, pl, grid, dev_err, st, pdl); \
        case kEpiBias: return launch_tile_one<XT, YT, kEpiBias, false>(a, tmq, tms, pl, grid, dev_err, st, pdl); \
        case kEpiBiasGelu:                                                                                       \
            return launch_tile_one<XT, YT, kEpiBiasGelu, false>(a, tmq, tms, pl, grid, dev_err, st, pdl);        \
        case kEpiBiasRes:                                                                                        \
            return launch_tile_one<XT, YT, kEpiBiasRes, false>(a, tmq, tms, pl, grid, dev_err, st, pdl);         \
        default: return cudaErrorInvalidValue;                                                                   \
    }
#define MADI_TILE_R16(YT)                                                                                           \
    switch (epi) {                                                                                                  \
        case kEpiNone: return launch_tile_one<float, YT, kEpiNone, false, true>(a, tmq, tms, pl, grid, dev_err, st, pdl); \
        case kEpiBias: return launch_tile_one<float, YT, kEpiBias, false, true>(a, tmq, tms, pl, grid, dev_err, st, pdl); \
        case kEpiBiasGelu:                                                                                          \
            return launch_tile_one<float, YT, kEpiBiasGelu, false, true>(a, tmq, tms, pl, grid, dev_err, st, pdl);   \
        case kEpiBiasRes:                                                                                           \
            return launch_tile_one<float, YT, kEpiBiasRes, false, true>(a, tmq, tms, pl, grid, dev_err, st, pdl);    \
        default: return cudaErrorInvalidValue;                                                                      \
    }
    if (x_r16 && y_f32) { MADI_TILE_R16(float) }
    if (x_r16) { MADI_TILE_R16(__half) }
#undef MADI_TILE_R16
    if (x_f32 && y_f32) { MADI_TILE_CASE(float, float) }
    if (x_f32 && !y_f32) { MADI_TILE_CASE(float, __half) }
    if (!x_f32 && y_f32) { MADI_TILE_CASE(__half, float) }
    MADI_TILE_CASE(__half, __half)
#undef MADI_TILE_CASE
}

}  // namespace madi
