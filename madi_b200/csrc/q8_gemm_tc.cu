// q8_gemm_tc.cu -- variant (a): Q8_0 linear on the 5th-generation tensor cores.
//
//   Y[m][n] = epi( sum_k X[m][k] * half(q[n][k] * s[n][k/32]) ),  f32 accumulate
//
// Semantics follow the reference's encoder path (kDeq + m4_gemm_*,
// encoder.zig:262-304): weights are dequantised to f16 with ONE rounding
// (q8_gemm.metal:25-26), products accumulate in f32, the epilogue adds the f32
// bias, applies the A&S GELU or adds the residual, and rounds once to f16.
//
// Design (one persistent CTA per SM, warp-specialised):
//   * the GEMM is computed transposed, Y^T = Wdq * X^T, so the DEQUANTISED
//     WEIGHT TILE is the MMA's A operand and lives in tensor memory: dequant
//     warps read int8 from shared memory, convert in registers and write f16
//     pairs straight to TMEM with tcgen05.st.  f16 weights never touch shared
//     memory or HBM.
//   * X tiles are the B operand: TMA (SWIZZLE_128B, no multicast) into shared
//     memory, read by tcgen05.mma through a K-major smem descriptor.
//   * int8 weight tiles arrive by TMA too (SWIZZLE_64B, conflict-free rows).
//   * the f32 accumulator (128 weight rows x BT tokens) sits in TMEM, double
//     buffered so the epilogue of tile i overlaps the MMAs of tile i+1.
//
// Warp roles (640 threads): w0 TMA producer, w1 MMA issuer + TMEM owner,
// w2-3 idle, w4-11 dequant in two groups of four that take alternate stages
// (TMEM lane quarter = warp % 4), w12-19 epilogue (two warps per lane quarter,
// each taking every second 32-token chunk of the accumulator).
// TMEM columns: [0, 2*BT) accumulators, then A_STAGES x 32 columns of A.  The
// shared-memory ring (X + int8 W per 64-K stage) is decoupled from the TMEM A
// ring and as deep as ~192 KB allows (6 stages at BT=192, 8 at BT=128), so TMA
// latency from L2/HBM is covered by bytes in flight.
// Every mbarrier wait is bounded; on expiry the CTA raises its abort flag,
// records the device error word, drains its in-flight copies and MMAs,
// frees TMEM and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "internal.h"

namespace madi {
namespace {

constexpr int BN = 128;        // weight rows per tile = MMA M
constexpr int BK = 64;         // K per pipeline stage
constexpr int A_STAGES = 4;    // TMEM ring of dequantised A stages (one-CTA kernel)
constexpr int MAX_A_STAGES = 8;
constexpr int MAX_STAGES = 8;  // shared-memory ring depth upper bound
constexpr int RING_BYTES = 192 * 1024;      // shared-memory ring budget (X + W stages)
constexpr int Y_ROWS = 32;                 // tokens per epilogue chunk
constexpr int Y_BUF = Y_ROWS * 128 * 2;    // one f16 [32 tokens][128 features] staging tile
constexpr int Y_STAGE_BYTES = 2 * 2 * Y_BUF;   // two epilogue halves x double buffer
constexpr int W_STAGE = BN * BK;           // int8 bytes
constexpr int A_STAGE_COLS = BK / 2;       // f16 pairs per TMEM column
constexpr int TMEM_COLS = 512;
constexpr int kDqWarp0 = 4;                // warps 4..11: dequant (two groups of four)
constexpr int kEpiWarp0 = 12;              // warps 12..19: epilogue
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);

static_assert(BK == 64, "umma_stage4_ts issues four K=16 MMAs per stage");

constexpr size_t kBarsBytes = 512;          // shared memory reserved for struct Bars (checked below)


template <int BT> struct Cfg {
    static constexpr int X_STAGE = BT * BK * 2;   // f16 bytes
    // as many shared-memory stages as the ring budget holds: DRAM/L2 latency is
    // covered by bytes in flight, so the ring is as deep as shared memory allows
    static constexpr int STAGES = RING_BYTES / (X_STAGE + W_STAGE) < MAX_STAGES
                                      ? RING_BYTES / (X_STAGE + W_STAGE) : MAX_STAGES;
    static constexpr int ACC_COLS = BT;
    static constexpr int A_COL0 = 2 * BT;
    static_assert(A_COL0 + A_STAGES * A_STAGE_COLS <= TMEM_COLS, "TMEM budget");
    static_assert(BT % 32 == 0 && BT >= 32 && BT <= 256, "MMA N");
    static_assert(STAGES >= 2, "ring depth");
    static constexpr uint32_t IDESC = idesc_f16_f32(BN, BT);
    static constexpr size_t SMEM_BASE = 1024 + (size_t)STAGES * (X_STAGE + W_STAGE) + kBarsBytes;
    static_assert(SMEM_BASE + Y_STAGE_BYTES <= 227 * 1024, "shared memory");
};

struct __align__(8) Bars {
    uint64_t full[MAX_STAGES];   // TMA bytes landed (X + W)
    uint64_t empty[MAX_STAGES];  // MMAs of the stage done (tcgen05.commit): X and W both consumed
    uint64_t aready[MAX_A_STAGES];   // dequantised A written to TMEM (one dequant group)
    uint64_t aempty[MAX_A_STAGES];   // MMAs reading the TMEM A stage done (tcgen05.commit)
    // Pair mode (even KT): the MMA thread takes two stages at a time, so readiness
    // and release are tracked per pair of stages -- half the barrier traffic on
    // the single MMA-issuing thread.
    uint64_t empty2[MAX_STAGES / 2];  // both smem stages of a pair consumed (tcgen05.commit)
    uint64_t aready2[MAX_A_STAGES / 2];   // both A stages of a pair written (both dequant groups)
    uint64_t aempty2[MAX_A_STAGES / 2];   // both A stages of a pair reusable (tcgen05.commit)
    uint64_t accfull[2];       // accumulator ready (tcgen05.commit)
    uint64_t accempty[2];      // epilogue drained the accumulator (one arrival per epilogue thread)
    uint64_t drain;            // final MMA drain
    uint32_t tmem_base;
    int abort;
};

static_assert(sizeof(Bars) <= kBarsBytes, "Bars must fit the shared memory reserved for it");

// Bounded wait that ignores the abort flag (used to drain in-flight work).
MADI_DEV void mbar_wait_drain(uint64_t *bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitBudgetCycles) return;
}

// 32 consecutive tokens (m) of one output feature (n): y[m][n] for m in [mb, mb+32).
template <int EPI>
MADI_DEV void epilogue_chunk(const GemmArgs &p, const uint32_t (&v)[32], int mb, int n, float bias) {
    const int N = p.N;
    const size_t base = (size_t)mb * N + n;
    if constexpr (EPI == kEpiNoneF32) {
        float *yf = reinterpret_cast<float *>(p.y);
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (mb + i < p.M) yf[base + (size_t)i * N] = __uint_as_float(v[i]);
        return;
    }
    if constexpr (EPI == kEpiResF32) {
        // x += half(acc) + bias in the reference's order ((x + mo) + bias); the
        // residual reads of each half chunk are issued together before its stores
        float *yf = reinterpret_cast<float *>(p.y);
        const float *rf = reinterpret_cast<const float *>(p.residual);
        const int nr = p.M - mb < 32 ? p.M - mb : 32;
#pragma unroll
        for (int hh = 0; hh < 32; hh += 16) {
            float r[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = hh + i < nr ? rf[base + (size_t)(hh + i) * N] : 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float mo = __half2float(__float2half_rn(__uint_as_float(v[hh + i])));
                if (hh + i < nr) yf[base + (size_t)(hh + i) * N] = __fadd_rn(__fadd_rn(r[i], mo), bias);
            }
        }
        return;
    }
    if (mb + 32 <= p.M) {
        float res[32];
        if constexpr (EPI == kEpiBiasRes) {
#pragma unroll
            for (int i = 0; i < 32; ++i) res[i] = __half2float(static_cast<const __half *>(p.residual)[base + (size_t)i * N]);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            float y = __uint_as_float(v[i]);
            if constexpr (EPI == kEpiBias) y += bias;
            if constexpr (EPI == kEpiBiasGelu) y = gelu_erf(y + bias);
            if constexpr (EPI == kEpiBiasRes) y = y + bias + res[i];
            p.y[base + (size_t)i * N] = __float2half_rn(y);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (mb + i < p.M) {
                float y = __uint_as_float(v[i]);
                if constexpr (EPI == kEpiBias) y += bias;
                if constexpr (EPI == kEpiBiasGelu) y = gelu_erf(y + bias);
                if constexpr (EPI == kEpiBiasRes)
                    y = y + bias + __half2float(static_cast<const __half *>(p.residual)[base + (size_t)i * N]);
                p.y[base + (size_t)i * N] = __float2half_rn(y);
            }
        }
    }
}

// 32 consecutive tokens of one feature into the staging tile: col[i * 128] =
// y[mb + i][n].  Rows past M / features past N are computed from zero-filled
// operands and clipped by the TMA store; residual reads stay in bounds.
template <int EPI>
MADI_DEV void epilogue_chunk_stage(const GemmArgs &p, const uint32_t (&v)[32], int mb, int n, float bias, bool nok,
                                   __half *col) {
    float res[32];
    if constexpr (EPI == kEpiBiasRes) {
        const size_t base = (size_t)mb * p.N + n;
#pragma unroll
        for (int i = 0; i < 32; ++i)
            res[i] = (nok && mb + i < p.M) ? __half2float(static_cast<const __half *>(p.residual)[base + (size_t)i * p.N])
                                           : 0.f;
    }
    if constexpr (EPI == kEpiBiasGelu) {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
            float a0, a1, y0, y1;
            add2(a0, a1, __uint_as_float(v[i]), __uint_as_float(v[i + 1]), bias, bias);
            gelu_erf2(y0, y1, a0, a1);
            col[i * BN] = __float2half_rn(y0);
            col[(i + 1) * BN] = __float2half_rn(y1);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            float y = __uint_as_float(v[i]);
            if constexpr (EPI == kEpiBias) y += bias;
            if constexpr (EPI == kEpiBiasRes) y = y + bias + res[i];
            col[i * BN] = __float2half_rn(y);
        }
    }
}

// Output staging (shared memory + TMA store) for the epilogues without a residual
// read.  The residual epilogue keeps direct stores and the smaller shared-memory
// footprint: measured faster for fc2, whose scale reads profit from the larger
// L1 left beside it.
template <int EPI> constexpr bool kStagedY = EPI != kEpiBiasRes && EPI != kEpiNoneF32 && EPI != kEpiResF32;
template <int BT, int EPI> constexpr size_t gemm_smem() {
    return Cfg<BT>::SMEM_BASE + (kStagedY<EPI> ? Y_STAGE_BYTES : 0);
}

template <int BT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    q8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                      const __grid_constant__ CUtensorMap tmY, const GemmArgs p, int ystore) {
    using C = Cfg<BT>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *xs = smem;
    uint8_t *ws = smem + STAGES * C::X_STAGE;
    uint8_t *ystage = ws + STAGES * W_STAGE;
    Bars *bars = reinterpret_cast<Bars *>(ystage + (kStagedY<EPI> ? Y_STAGE_BYTES : 0));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = p.M, N = p.N, K = p.K;
    const int n_tiles = (N + BN - 1) / BN;
    const int num_tiles = n_tiles * ((M + BT - 1) / BT);
    const int KT = (K + BK - 1) / BK;
    const int nkb = K / 32;
    // pair mode: KT, STAGES and A_STAGES even, so a pair of stages never wraps a
    // ring or spans two tiles
    const bool pairs = (KT & 1) == 0 && (STAGES & 1) == 0 && (A_STAGES & 1) == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < A_STAGES; ++a) {
            mbar_init(&bars->aready[a], 128);
            mbar_init(&bars->aempty[a], 1);
        }
        for (int i = 0; i < MAX_STAGES / 2; ++i) mbar_init(&bars->empty2[i], 1);
        for (int i = 0; i < A_STAGES / 2; ++i) {
            mbar_init(&bars->aready2[i], 256);
            mbar_init(&bars->aempty2[i], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->accfull[b], 1);
            mbar_init(&bars->accempty[b], kEpiWarps * 32);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    volatile int *abort_flag = &bars->abort;
    int *err = p.dev_err;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            uint32_t issued_mask = 0, last_ph[STAGES];
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                const int m0 = (tile / n_tiles) * BT, n0 = (tile % n_tiles) * BN;
                for (int kt = 0; kt < KT; ++kt) {
                    if (!mbar_wait(pairs ? &bars->empty2[s >> 1] : &bars->empty[s], ph ^ 1, abort_flag, err))
                        goto producer_done;
                    mbar_arrive_expect_tx(&bars->full[s], C::X_STAGE + W_STAGE);
                    tma_load_2d(xs + s * C::X_STAGE, &tmX, &bars->full[s], kt * BK, m0);
                    tma_load_2d(ws + s * W_STAGE, &tmW, &bars->full[s], kt * BK, n0);
                    issued_mask |= 1u << s;
                    last_ph[s] = ph;
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
            }
        producer_done:
            // the copies issued last must land before shared memory is released
            for (int i = 0; i < STAGES; ++i)
                if (issued_mask & (1u << i)) mbar_wait_drain(&bars->full[i], last_ph[i]);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            int s = 0, a = 0, lt = 0;
            uint32_t ph = 0, pha = 0;
            // Everything a stage's MMAs need is advanced by adds: the B descriptor's
            // low word (start address in 16-byte units), the A columns and the two
            // commit barriers.  The MMA thread shares its scheduler with four busy
            // warps, so its per-stage instruction count bounds the MMA issue rate.
            const uint64_t desc0 = smem_desc_sw128(smem_u32(xs));
            const uint32_t desc_hi = (uint32_t)(desc0 >> 32);
            const uint32_t desc_lo0 = (uint32_t)desc0;
            constexpr uint32_t kDescStep = C::X_STAGE >> 4;
            const uint32_t empty0 = smem_u32(&bars->empty[0]), aempty0 = smem_u32(&bars->aempty[0]);
            const uint32_t a_tmem0 = tmem + C::A_COL0;
            const uint32_t empty2_0 = smem_u32(&bars->empty2[0]), aempty2_0 = smem_u32(&bars->aempty2[0]);
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
                const int b = lt & 1;
                const uint32_t aph = (lt >> 1) & 1;
                if (!mbar_wait(&bars->accempty[b], aph ^ 1, abort_flag, err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + b * C::ACC_COLS;
                bool ok = true;
                if (pairs) {
                    // two stages per iteration (s and a stay even): one readiness wait and
                    // two release commits per pair; pair slot a / 2, phase pha
                    for (int kt = 0; kt < KT; kt += 2) {
                        if (!mbar_wait(&bars->aready2[a >> 1], pha, abort_flag, err)) { ok = false; break; }
                        tc_fence_after();
                        umma_stage8_ts_2c(d_tmem, a_tmem0 + a * A_STAGE_COLS, desc_lo0 + (uint32_t)s * kDescStep,
                                          desc_hi, kDescStep, C::IDESC, kt != 0, empty2_0 + 8u * (s >> 1),
                                          aempty2_0 + 8u * (a >> 1));
                        if ((s += 2) == STAGES) { s = 0; ph ^= 1; }
                        if ((a += 2) == A_STAGES) { a = 0; pha ^= 1; }
                    }
                } else {
                    for (int kt = 0; kt < KT; ++kt) {
                        if (!mbar_wait(&bars->aready[a], pha, abort_flag, err)) { ok = false; break; }
                        tc_fence_after();
                        // X (MMA) and W (dequant, earlier) of smem stage s consumed; TMEM A stage a reusable
                        umma_stage4_ts(d_tmem, a_tmem0 + a * A_STAGE_COLS, desc_lo0 + (uint32_t)s * kDescStep, desc_hi,
                                       C::IDESC, kt != 0, empty0 + 8u * s, aempty0 + 8u * a);
                        if (++s == STAGES) { s = 0; ph ^= 1; }
                        if (++a == A_STAGES) { a = 0; pha ^= 1; }
                    }
                }
                if (!ok) break;
                umma_commit(&bars->accfull[b]);
            }
            // every MMA issued must finish before TMEM is released
            umma_commit(&bars->drain);
            mbar_wait_drain(&bars->drain, 0);
        }
        __syncwarp();
    } else if (warp >= kDqWarp0 && warp < kEpiWarp0) {
        // ------------------------------------------------ dequant: int8 smem -> f16 TMEM
        // Two groups of four warps take alternate pipeline stages; within a
        // group, warp % 4 selects the TMEM lane quarter and lane = weight row.
        const int grp = (warp - kDqWarp0) >> 2;
        const int q = warp & 3;
        const int r = q * 32 + lane;            // weight row within the tile = TMEM lane
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        const int swz = (r >> 1) & 3;           // SWIZZLE_64B: 16-byte chunk c lives at c ^ swz
        const bool pair_ok = (nkb & 1) == 0;    // both block scales of a stage in one aligned word
        const int gstep = (int)(gridDim.x % (unsigned)n_tiles);

        // A cursor over this group's stages (every second one): the tile, its
        // row-block index and the k-step, advanced without divisions.
        struct Cur {
            int kt, tile, nt;
        };
        auto adv = [&](Cur &c) {
            c.kt += 2;
            while (c.kt >= KT) {
                c.kt -= KT;
                c.tile += gridDim.x;
                c.nt += gstep;
                if (c.nt >= n_tiles) c.nt -= n_tiles;
            }
        };
        // f16 scale pair (blocks 2kt, 2kt+1) of this thread's row at cursor c.  The
        // loads are predicated PTX loads whose destinations nothing reads until the
        // stage that uses them, so their L2 latency overlaps the two visits in
        // between (a select on the loaded value here would stall).
        auto scale_at = [&](const Cur &c) -> uint2 {
            const int n = c.nt * BN + r;
            const int kb = 2 * c.kt;
            const bool rowok = c.tile < num_tiles && n < N;
            const __half *sp = p.scales + (size_t)(rowok ? n : 0) * nkb + (rowok ? kb : 0);
            uint2 v = make_uint2(0u, 0u);
            if (pair_ok) {
                ldg_nc_u32_pred(v.x, sp, rowok);
            } else {
                ldg_nc_u16_pred(v.x, sp, rowok && kb < nkb);
                ldg_nc_u16_pred(v.y, sp + 1, rowok && kb + 1 < nkb);
            }
            return v;
        };
        // ring positions of the stage being visited (smem ring s/ph, TMEM A ring as/pha)
        int s = grp % STAGES, as = grp % A_STAGES;
        uint32_t ph = (uint32_t)(grp / STAGES) & 1u, pha = (uint32_t)(grp / A_STAGES) & 1u;
        // dequantise the visited stage (tile `tile`) with scale pair `swv`; false when
        // done or aborted
        auto visit = [&](int tile, uint2 swv) -> bool {
            if (tile >= num_tiles) return false;
            // convert as soon as the int8 stage has landed, then wait for the TMEM
            // slot: the conversion stays off the MMA -> dequant -> MMA round trip
            if (!warp_wait_all(&bars->full[s], ph, abort_flag, err)) return false;
            const uint32_t sw = pair_ok ? swv.x : (swv.x | (swv.y << 16));
            const __half2 sw2 = *reinterpret_cast<const __half2 *>(&sw);
            const __half2 sc_lo = __low2half2(sw2), sc_hi = __high2half2(sw2);
            const uint8_t *wrow = ws + s * W_STAGE + r * 64;
            uint32_t a[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 v = *reinterpret_cast<const uint4 *>(wrow + ((c ^ swz) << 4));
                const __half2 sc = c < 2 ? sc_lo : sc_hi;
                const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    __half2 lo, hi;
                    q8_to_half2x2(wv[i], lo, hi);
                    a[c * 8 + 2 * i] = h2_as_u32(__hmul2(lo, sc));      // half(q*s): one rounding
                    a[c * 8 + 2 * i + 1] = h2_as_u32(__hmul2(hi, sc));
                }
            }
            if (!warp_wait_all(pairs ? &bars->aempty2[as >> 1] : &bars->aempty[as], pha ^ 1u, abort_flag, err))
                return false;
            tc_fence_after();
            tmem_st32(tmem + lane_addr + C::A_COL0 + as * A_STAGE_COLS, a);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(pairs ? &bars->aready2[as >> 1] : &bars->aready[as]);
            s += 2;
            if (s >= STAGES) { s -= STAGES; ph ^= 1u; }
            as += 2;
            if (as >= A_STAGES) { as -= A_STAGES; pha ^= 1u; }
            return true;
        };
        // this group visits stages grp, grp+2, ...; scales are fetched two visits
        // (four stages) ahead so their L2 latency is off the critical path
        Cur vc{grp % KT, (int)blockIdx.x + (grp / KT) * (int)gridDim.x, 0};
        vc.nt = vc.tile % n_tiles;
        Cur pc = vc;
        adv(pc);
        uint2 sA = scale_at(vc), sB = scale_at(pc);
        adv(pc);                                // prefetch cursor: four stages ahead
        while (true) {
            uint2 use = sA;
            sA = scale_at(pc);
            adv(pc);
            if (!visit(vc.tile, use)) break;
            adv(vc);
            use = sB;
            sB = scale_at(pc);
            adv(pc);
            if (!visit(vc.tile, use)) break;
            adv(vc);
        }
    } else if (warp >= kEpiWarp0) {
        // ------------------------------------------------ epilogue: TMEM -> bias/GELU/residual -> f16
        const int q = warp & 3;
        const int half = (warp - kEpiWarp0) >> 2;   // which of the two warps of lane quarter q
        const int r = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        // With ystore, each half stages its 32-token chunks (all 128 features: the
        // four warps of the half) in shared memory and one thread writes the chunk
        // with a TMA store; the two staging tiles of a half alternate.
        const bool leader = q == 0 && lane == 0;
        const int bar_id = 1 + half;
        uint8_t *ybuf = ystage + half * 2 * Y_BUF;
        int ycnt = 0;
        int lt = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
            const int b = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!warp_wait_all(&bars->accfull[b], aph, abort_flag, err)) break;
            tc_fence_after();
            const int m0 = (tile / n_tiles) * BT;
            const int n0 = (tile % n_tiles) * BN;
            const int n = n0 + r;
            const bool nok = n < N;
            float bias = 0.f;
            if constexpr (EPI != kEpiNone && EPI != kEpiNoneF32) {      // kEpiResF32 has a bias
                if (nok)
                    bias = p.bias_f16 ? __half2float(reinterpret_cast<const __half *>(p.bias)[n])
                                      : reinterpret_cast<const float *>(p.bias)[n];
            }
            const uint32_t acc_addr = tmem + lane_addr + b * C::ACC_COLS;
            // load -> wait -> use: no register written by an in-flight tcgen05.ld is
            // ever live across compiler-scheduled code
#pragma unroll 1
            for (int c = half; c < BT / 32; c += 2) {
                uint32_t v[32];
                tmem_ld32(acc_addr + c * 32, v);
                tmem_wait_ld();
                if (kStagedY<EPI> && ystore) {
                    __half *buf = reinterpret_cast<__half *>(ybuf + (ycnt & 1) * Y_BUF);
                    if (leader) bulk_wait_group_read<1>();   // the store that last used buf has read it
                    named_bar_sync(bar_id, 128);
                    epilogue_chunk_stage<EPI>(p, v, m0 + c * 32, n, bias, nok, buf + r);
                    fence_proxy_async_smem();
                    named_bar_sync(bar_id, 128);
                    if (leader) {
                        tma_store_2d(&tmY, buf, n0, m0 + c * 32);
                        bulk_commit_group();
                    }
                    ++ycnt;
                } else if (nok) {
                    epilogue_chunk<EPI>(p, v, m0 + c * 32, n, bias);
                }
            }
            tc_fence_before();
            mbar_arrive(&bars->accempty[b]);
        }
        if (leader) bulk_wait_group_all();   // stores complete before shared memory goes away
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <int BT, int EPI>
cudaError_t launch_bt(const GemmArgs &a, const CUtensorMap &tmX, const CUtensorMap &tmW, const CUtensorMap &tmY,
                      int ystore, int num_sms, cudaStream_t st) {
    using C = Cfg<BT>;
    auto fn = q8_gemm_tc_kernel<BT, EPI>;
    // once per instantiation: launches inside a capture stay pure launches
    static std::once_flag once;
    static cudaError_t once_status;
    if (cudaError_t e = run_once(once, once_status, [&] {
            return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem<BT, EPI>());
        }))
        return e;
    const int tiles = ((a.N + BN - 1) / BN) * ((a.M + BT - 1) / BT);
    const int grid = tiles < num_sms ? tiles : num_sms;
    fn<<<grid, kThreads, gemm_smem<BT, EPI>(), st>>>(tmX, tmW, tmY, a, ystore);
    return cudaGetLastError();
}

// ================================================================ CTA-pair kernel
//
// The same pipeline on a cluster of two CTAs sharing every MMA (cta_group::2,
// M = 256): a pair tile is 256 weight rows x 192 tokens.  Each CTA dequantises
// its own 128 weight rows into its own tensor memory (A rows 0-127 in the even
// CTA, 128-255 in the odd one) and stages its own 96-token half of the X tile
// (B columns 0-95 in the even CTA, 96-191 in the odd one); the even CTA's MMA
// thread issues the pair's MMAs, and each CTA's accumulator holds its 128
// weight rows x all 192 tokens, which its own epilogue warps write out.
// Compared with one CTA per tile this halves, per SM, the MMA instructions,
// barrier waits and commits the single issuing thread handles, and the X bytes
// each SM stages from L2.
//
// Synchronisation across the pair:
//   * full[s]   (each CTA): its own TMA bytes (X half + int8 W) landed;
//   * aready*   (even CTA): both CTAs' dequant warps wrote the A stage(s) --
//               one arrival per warp, after tcgen05.wait::st and
//               tcgen05.fence::before_thread_sync (a cluster-scope release on
//               these arrivals was measured to cost 40 % of the kernel time);
//   * empty*, aempty*, accfull, drain (each CTA): tcgen05.commit multicast to
//               both CTAs by the even CTA's MMA thread;
//   * accempty  (even CTA): both CTAs' epilogue warps drained the accumulator.
// Both CTAs pass a cluster barrier after initialising their barriers and
// before the first remote arrival, and again before tensor memory is freed and
// the CTAs exit, so no arrival or MMA ever targets a CTA that has left.  A
// bounded wait that expires raises the abort flag of both CTAs.
constexpr int PBN = 2 * BN;       // weight rows per pair tile (MMA M)

// PBT tokens per pair tile (MMA N; each CTA stages PBT / 2 of them).  The A
// ring takes the tensor-memory columns the two accumulators leave: 4 stages at
// PBT = 192 and two at 224.  Narrower tiles (deeper A rings: 6 stages at 160, 8 at
// 128) were measured slower, 941 and 830 TFLOP/s against 1035 on the encoder FFN
// pair; 224 measured 1047 against 1025 at 192 there (fc1 3.8 % faster).
constexpr int kPairTokens = 192;
constexpr int kPairTokensWide = 224;     // the wider tile, chosen per shape by pair_tokens()
template <int PBT> struct PCfg {
    static constexpr int PHALF = PBT / 2;
    static constexpr int X_STAGE = PHALF * BK * 2;   // f16 bytes of one CTA's X half
    static constexpr int STAGES = RING_BYTES / (X_STAGE + W_STAGE) < MAX_STAGES
                                      ? RING_BYTES / (X_STAGE + W_STAGE) : MAX_STAGES;
    static constexpr int ACC_COLS = PBT;
    static constexpr int A_COL0 = 2 * PBT;
    static constexpr int A_ST_RAW = (TMEM_COLS - A_COL0) / A_STAGE_COLS;
    static constexpr int A_ST = (A_ST_RAW > MAX_A_STAGES ? MAX_A_STAGES : A_ST_RAW) & ~1;
    static_assert(A_ST >= 2 && A_COL0 + A_ST * A_STAGE_COLS <= TMEM_COLS, "TMEM budget");
    static_assert(STAGES % 2 == 0, "pair mode needs an even ring");
    static_assert(X_STAGE % 1024 == 0, "SWIZZLE_128B atoms");
    static_assert(PBT % 32 == 0 && PBT >= 64 && PBT <= 256, "MMA N");
    static constexpr uint32_t IDESC = idesc_f16_f32(PBN, PBT);
    static constexpr size_t SMEM_BASE = 1024 + (size_t)STAGES * (X_STAGE + W_STAGE) + kBarsBytes;
    static_assert(SMEM_BASE + Y_STAGE_BYTES <= 227 * 1024, "shared memory");
};
constexpr int kPairDqArrivals = 2 * 4;         // dequant warps of one stage, both CTAs
constexpr int kPairEpiArrivals = 2 * kEpiWarps; // epilogue warps, both CTAs

template <int PBT, int EPI> constexpr size_t pair_smem() {
    return PCfg<PBT>::SMEM_BASE + (kStagedY<EPI> ? Y_STAGE_BYTES : 0);
}

template <int PBT, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    q8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ CUtensorMap tmY, const GemmArgs p, int ystore) {
    using C = PCfg<PBT>;
    constexpr int STAGES = C::STAGES;
    constexpr int A_STAGES = C::A_ST;
    constexpr int PHALF = C::PHALF;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *xs = smem;
    uint8_t *ws = smem + STAGES * C::X_STAGE;
    uint8_t *ystage = ws + STAGES * W_STAGE;
    Bars *bars = reinterpret_cast<Bars *>(ystage + (kStagedY<EPI> ? Y_STAGE_BYTES : 0));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();        // 0: issues the pair's MMAs
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    const int M = p.M, N = p.N, K = p.K;
    const int n_tiles = (N + PBN - 1) / PBN;
    const int num_tiles = n_tiles * ((M + PBT - 1) / PBT);
    const int KT = (K + BK - 1) / BK;
    const int nkb = K / 32;
    // pair mode issues two K stages per MMA-thread step; it needs two pairs of TMEM A
    // stages so the dequant of one pair overlaps the MMAs of the other
    const bool pairs = (KT & 1) == 0 && A_STAGES >= 4;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < A_STAGES; ++a) {
            mbar_init(&bars->aready[a], kPairDqArrivals);
            mbar_init(&bars->aempty[a], 1);
        }
        for (int i = 0; i < MAX_STAGES / 2; ++i) mbar_init(&bars->empty2[i], 1);
        for (int i = 0; i < A_STAGES / 2; ++i) {
            mbar_init(&bars->aready2[i], 2 * kPairDqArrivals);
            mbar_init(&bars->aempty2[i], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->accfull[b], 1);
            mbar_init(&bars->accempty[b], kPairEpiArrivals);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
    }
    if (warp == 1) {
        tmem_alloc2(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish2();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();      // the peer's barriers are initialised before any arrival reaches them
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    volatile int *abort_flag = &bars->abort;
    const uint32_t peer_abort = mapa_u32(&bars->abort, rank ^ 1u);
    int *err = p.dev_err;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (each CTA: its X half + its W rows)
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            uint32_t issued_mask = 0, last_ph[STAGES];
            for (int tile = pair; tile < num_tiles; tile += npairs) {
                const int m0 = (tile / n_tiles) * PBT + (int)rank * PHALF;
                const int n0 = (tile % n_tiles) * PBN + (int)rank * BN;
                for (int kt = 0; kt < KT; ++kt) {
                    if (!mbar_wait_cl(pairs ? &bars->empty2[s >> 1] : &bars->empty[s], ph ^ 1, abort_flag, peer_abort,
                                      err))
                        goto producer_done;
                    mbar_arrive_expect_tx(&bars->full[s], C::X_STAGE + W_STAGE);
                    tma_load_2d(xs + s * C::X_STAGE, &tmX, &bars->full[s], kt * BK, m0);
                    tma_load_2d(ws + s * W_STAGE, &tmW, &bars->full[s], kt * BK, n0);
                    issued_mask |= 1u << s;
                    last_ph[s] = ph;
                    if (++s == STAGES) { s = 0; ph ^= 1; }
                }
            }
        producer_done:
            for (int i = 0; i < STAGES; ++i)
                if (issued_mask & (1u << i)) mbar_wait_drain(&bars->full[i], last_ph[i]);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (even CTA only)
        if (rank == 0 && lane == 0) {
            int s = 0, a = 0, lt = 0;
            uint32_t pha = 0;
            const uint64_t desc0 = smem_desc_sw128(smem_u32(xs));
            const uint32_t desc_hi = (uint32_t)(desc0 >> 32);
            const uint32_t desc_lo0 = (uint32_t)desc0;
            constexpr uint32_t kDescStep = C::X_STAGE >> 4;
            const uint32_t empty0 = smem_u32(&bars->empty[0]), aempty0 = smem_u32(&bars->aempty[0]);
            const uint32_t empty2_0 = smem_u32(&bars->empty2[0]), aempty2_0 = smem_u32(&bars->aempty2[0]);
            const uint32_t a_tmem0 = tmem + C::A_COL0;
            for (int tile = pair; tile < num_tiles; tile += npairs, ++lt) {
                const int b = lt & 1;
                const uint32_t aph = (lt >> 1) & 1;
                if (!mbar_wait_cl(&bars->accempty[b], aph ^ 1, abort_flag, peer_abort, err)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + b * C::ACC_COLS;
                bool ok = true;
                if (pairs) {
                    for (int kt = 0; kt < KT; kt += 2) {
                        if (!mbar_wait_cl(&bars->aready2[a >> 1], pha, abort_flag, peer_abort, err)) { ok = false; break; }
                        tc_fence_after();
                        umma2_stage8_ts_2c(d_tmem, a_tmem0 + a * A_STAGE_COLS, desc_lo0 + (uint32_t)s * kDescStep,
                                           desc_hi, kDescStep, C::IDESC, kt != 0, empty2_0 + 8u * (s >> 1),
                                           aempty2_0 + 8u * (a >> 1));
                        if ((s += 2) == STAGES) s = 0;
                        if ((a += 2) == A_STAGES) { a = 0; pha ^= 1; }
                    }
                } else {
                    for (int kt = 0; kt < KT; ++kt) {
                        if (!mbar_wait_cl(&bars->aready[a], pha, abort_flag, peer_abort, err)) { ok = false; break; }
                        tc_fence_after();
                        umma2_stage4_ts(d_tmem, a_tmem0 + a * A_STAGE_COLS, desc_lo0 + (uint32_t)s * kDescStep, desc_hi,
                                        C::IDESC, kt != 0, empty0 + 8u * s, aempty0 + 8u * a);
                        if (++s == STAGES) s = 0;
                        if (++a == A_STAGES) { a = 0; pha ^= 1; }
                    }
                }
                if (!ok) break;
                umma2_commit_both(&bars->accfull[b]);
            }
            // every MMA issued must finish before either CTA releases tensor memory
            umma2_commit_both(&bars->drain);
            mbar_wait_drain(&bars->drain, 0);
        }
        __syncwarp();
    } else if (warp >= kDqWarp0 && warp < kEpiWarp0) {
        // ------------------------------------------------ dequant: int8 smem -> f16 TMEM (this CTA's rows)
        const int grp = (warp - kDqWarp0) >> 2;
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        const int swz = (r >> 1) & 3;
        const bool pair_ok = (nkb & 1) == 0;
        const int gstep = npairs % n_tiles;
        const int rbase = (int)rank * BN + r;       // row within the pair tile
        const uint32_t aready0 = mapa_u32(&bars->aready[0], 0), aready2_0 = mapa_u32(&bars->aready2[0], 0);
        struct Cur {
            int kt, tile, nt;
        };
        auto adv = [&](Cur &c) {
            c.kt += 2;
            while (c.kt >= KT) {
                c.kt -= KT;
                c.tile += npairs;
                c.nt += gstep;
                if (c.nt >= n_tiles) c.nt -= n_tiles;
            }
        };
        auto scale_at = [&](const Cur &c) -> uint2 {
            const int n = c.nt * PBN + rbase;
            const int kb = 2 * c.kt;
            const bool rowok = c.tile < num_tiles && n < N;
            const __half *sp = p.scales + (size_t)(rowok ? n : 0) * nkb + (rowok ? kb : 0);
            uint2 v = make_uint2(0u, 0u);
            if (pair_ok) {
                ldg_nc_u32_pred(v.x, sp, rowok);
            } else {
                ldg_nc_u16_pred(v.x, sp, rowok && kb < nkb);
                ldg_nc_u16_pred(v.y, sp + 1, rowok && kb + 1 < nkb);
            }
            return v;
        };
        int s = grp % STAGES, as = grp % A_STAGES;
        uint32_t ph = (uint32_t)(grp / STAGES) & 1u, pha = (uint32_t)(grp / A_STAGES) & 1u;
        auto visit = [&](int tile, uint2 swv) -> bool {
            if (tile >= num_tiles) return false;
            if (!warp_wait_all_cl(&bars->full[s], ph, abort_flag, peer_abort, err)) return false;
            const uint32_t sw = pair_ok ? swv.x : (swv.x | (swv.y << 16));
            const __half2 sw2 = *reinterpret_cast<const __half2 *>(&sw);
            const __half2 sc_lo = __low2half2(sw2), sc_hi = __high2half2(sw2);
            const uint8_t *wrow = ws + s * W_STAGE + r * 64;
            uint32_t a[32];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 v = *reinterpret_cast<const uint4 *>(wrow + ((c ^ swz) << 4));
                const __half2 sc = c < 2 ? sc_lo : sc_hi;
                const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    __half2 lo, hi;
                    q8_to_half2x2(wv[i], lo, hi);
                    a[c * 8 + 2 * i] = h2_as_u32(__hmul2(lo, sc));
                    a[c * 8 + 2 * i + 1] = h2_as_u32(__hmul2(hi, sc));
                }
            }
            if (!warp_wait_all_cl(pairs ? &bars->aempty2[as >> 1] : &bars->aempty[as], pha ^ 1u, abort_flag, peer_abort,
                                  err))
                return false;
            tc_fence_after();
            tmem_st32(tmem + lane_addr + C::A_COL0 + as * A_STAGE_COLS, a);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(pairs ? aready2_0 + 8u * (as >> 1) : aready0 + 8u * as);
            s += 2;
            if (s >= STAGES) { s -= STAGES; ph ^= 1u; }
            as += 2;
            if (as >= A_STAGES) { as -= A_STAGES; pha ^= 1u; }
            return true;
        };
        Cur vc{grp % KT, pair + (grp / KT) * npairs, 0};
        vc.nt = vc.tile % n_tiles;
        Cur pc = vc;
        adv(pc);
        uint2 sA = scale_at(vc), sB = scale_at(pc);
        adv(pc);
        while (true) {
            uint2 use = sA;
            sA = scale_at(pc);
            adv(pc);
            if (!visit(vc.tile, use)) break;
            adv(vc);
            use = sB;
            sB = scale_at(pc);
            adv(pc);
            if (!visit(vc.tile, use)) break;
            adv(vc);
        }
    } else if (warp >= kEpiWarp0) {
        // ------------------------------------------------ epilogue: this CTA's 128 rows x 192 tokens
        const int q = warp & 3;
        const int half = (warp - kEpiWarp0) >> 2;
        const int r = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        const bool leader = q == 0 && lane == 0;
        const int bar_id = 1 + half;
        uint8_t *ybuf = ystage + half * 2 * Y_BUF;
        const uint32_t accempty0 = mapa_u32(&bars->accempty[0], 0);
        int ycnt = 0;
        int lt = 0;
        for (int tile = pair; tile < num_tiles; tile += npairs, ++lt) {
            const int b = lt & 1;
            const uint32_t aph = (lt >> 1) & 1;
            if (!warp_wait_all_cl(&bars->accfull[b], aph, abort_flag, peer_abort, err)) break;
            tc_fence_after();
            const int m0 = (tile / n_tiles) * PBT;
            const int n0 = (tile % n_tiles) * PBN + (int)rank * BN;
            const int n = n0 + r;
            const bool nok = n < N;
            float bias = 0.f;
            if constexpr (EPI != kEpiNone && EPI != kEpiNoneF32) {      // kEpiResF32 has a bias
                if (nok)
                    bias = p.bias_f16 ? __half2float(reinterpret_cast<const __half *>(p.bias)[n])
                                      : reinterpret_cast<const float *>(p.bias)[n];
            }
            const uint32_t acc_addr = tmem + lane_addr + b * C::ACC_COLS;
#pragma unroll 1
            for (int c = half; c < PBT / 32; c += 2) {
                uint32_t v[32];
                tmem_ld32(acc_addr + c * 32, v);
                tmem_wait_ld();
                if (kStagedY<EPI> && ystore) {
                    __half *buf = reinterpret_cast<__half *>(ybuf + (ycnt & 1) * Y_BUF);
                    if (leader) bulk_wait_group_read<1>();
                    named_bar_sync(bar_id, 128);
                    epilogue_chunk_stage<EPI>(p, v, m0 + c * 32, n, bias, nok, buf + r);
                    fence_proxy_async_smem();
                    named_bar_sync(bar_id, 128);
                    if (leader) {
                        tma_store_2d(&tmY, buf, n0, m0 + c * 32);
                        bulk_commit_group();
                    }
                    ++ycnt;
                } else if (nok) {
                    epilogue_chunk<EPI>(p, v, m0 + c * 32, n, bias);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(accempty0 + 8u * b);
        }
        if (leader) bulk_wait_group_all();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();      // no MMA, commit or arrival targets either CTA past this point
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc2(tmem, TMEM_COLS);
    }
}

template <int PBT, int EPI>
cudaError_t launch_pair(const GemmArgs &a, const CUtensorMap &tmX, const CUtensorMap &tmW, const CUtensorMap &tmY,
                        int ystore, int num_sms, cudaStream_t st) {
    auto fn = q8_gemm_pair_kernel<PBT, EPI>;
    static int max_pairs = 1;      // once per instantiation: co-resident clusters on this device
    static std::once_flag once;
    static cudaError_t once_status;
    if (cudaError_t e0 = run_once(once, once_status, [&] {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pair_smem<PBT, EPI>());
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (num_sms / 2));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = pair_smem<PBT, EPI>();
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, fn, &cfg);
        if (e != cudaSuccess) return e;
        max_pairs = n > 0 ? n : 1;
        return cudaSuccess;
    }))
        return e0;
    const int tiles = ((a.N + PBN - 1) / PBN) * ((a.M + PBT - 1) / PBT);
    const int pairs = tiles < max_pairs ? tiles : max_pairs;
    fn<<<2 * pairs, kThreads, pair_smem<PBT, EPI>(), st>>>(tmX, tmW, tmY, a, ystore);
    return cudaGetLastError();
}

bool make_map(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
    PFN_encodeTiled enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Token-tile width: the candidate with the lowest waves x (tile length + a fixed
// per-tile cost of 32 token columns) wins, the wider tile on ties (it amortises
// the weight dequant over more tokens).
int pick_bt(int M, int N, int num_sms) {
    const int n_tiles = (N + BN - 1) / BN;
    long best_cost = -1;
    int best = 192;
    for (int bt : {192, 128}) {
        const long tiles = (long)n_tiles * ((M + bt - 1) / bt);
        const long waves = (tiles + num_sms - 1) / num_sms;
        const long cost = waves * (bt + 32);
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = bt; }
    }
    return best;
}

}  // namespace

PFN_encodeTiled tensor_map_encoder() {
    static PFN_encodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled>(ptr);
    });
    return fn;
}

// CTA-pair kernel by default; MADI_GEMM_PAIR=0 in the environment selects the
// one-CTA kernel (kept for comparison and for devices without cluster support).
static bool use_pair_kernel() {
    static const bool v = [] {
        const char *e = getenv("MADI_GEMM_PAIR");
        return !(e && e[0] == '0');
    }();
    return v;
}
// Tokens per CTA-pair tile, 192 or 224.  A K stage costs about 2 (192 + tokens)
// cycles of the pair (measured over 128-224 token tiles), so the wider tile does
// 7 % more work per cycle; its 448 accumulator columns leave two TMEM A stages, so
// the MMA thread takes one K stage at a time.  The tile with the lower
// waves x (192 + tokens) wins, 192 on ties: 224 for the encoder FFN pair at 16
// chunks (fc1 30 waves against 34), 192 for shapes that fit one wave.
// MADI_GEMM_PBT=192 or 224 in the environment forces one (for comparisons).
static int pair_tokens(int M, int N, int num_sms) {
    static const int forced = [] {
        const char *e = getenv("MADI_GEMM_PBT");
        const int v = e ? atoi(e) : 0;
        return v == 192 || v == 224 ? v : 0;
    }();
    if (forced) return forced;
    const long pairs = num_sms / 2 > 0 ? num_sms / 2 : 1;
    const long n_tiles = (N + PBN - 1) / PBN;
    long best_cost = -1;
    int best = kPairTokens;
    for (int pbt : {kPairTokens, kPairTokensWide}) {
        const long waves = (n_tiles * ((M + pbt - 1) / pbt) + pairs - 1) / pairs;
        const long cost = waves * (192 + pbt);
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = pbt; }
    }
    return best;
}

template <int PBT>
static cudaError_t launch_pair_epi(const GemmArgs &a, int epi, const CUtensorMap &tmX, const CUtensorMap &tmW,
                                   const CUtensorMap &tmY, int ystore, int num_sms, cudaStream_t st) {
    switch (epi) {
        case kEpiNone: return launch_pair<PBT, kEpiNone>(a, tmX, tmW, tmY, ystore, num_sms, st);
        case kEpiBias: return launch_pair<PBT, kEpiBias>(a, tmX, tmW, tmY, ystore, num_sms, st);
        case kEpiBiasGelu: return launch_pair<PBT, kEpiBiasGelu>(a, tmX, tmW, tmY, ystore, num_sms, st);
        case kEpiBiasRes: return launch_pair<PBT, kEpiBiasRes>(a, tmX, tmW, tmY, ystore, num_sms, st);
        case kEpiNoneF32: return launch_pair<PBT, kEpiNoneF32>(a, tmX, tmW, tmY, 0, num_sms, st);
        case kEpiResF32: return launch_pair<PBT, kEpiResF32>(a, tmX, tmW, tmY, 0, num_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemm_tc(const GemmArgs &a, int epi, int num_sms, cudaStream_t st) {
    const bool pair = use_pair_kernel() && num_sms >= 2;
    const int pbt = pair ? pair_tokens(a.M, a.N, num_sms) : 0;
    const int bt = pair ? pbt / 2 : pick_bt(a.M, a.N, num_sms);   // X box rows
    CUtensorMap tmX, tmW;
    if (!make_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2, BK,
                  (uint32_t)bt, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorNotSupported;
    if (!make_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.qs, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, BK, BN,
                  CU_TENSOR_MAP_SWIZZLE_64B))
        return cudaErrorNotSupported;
    // Output through staged TMA stores when the row pitch allows a tensor map
    // (N * 2 bytes a multiple of 16); otherwise the epilogue stores directly.
    CUtensorMap tmY;
    int ystore = epi != kEpiNoneF32 && epi != kEpiResF32 && a.N % 8 == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 &&
                 make_map(&tmY, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.y, (uint64_t)a.N, (uint64_t)a.M,
                          (uint64_t)a.N * 2, BN, Y_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!ystore) memset(&tmY, 0, sizeof(tmY));
    if (pair)
        return pbt == kPairTokensWide ? launch_pair_epi<kPairTokensWide>(a, epi, tmX, tmW, tmY, ystore, num_sms, st)
                          : launch_pair_epi<kPairTokens>(a, epi, tmX, tmW, tmY, ystore, num_sms, st);
#define MADI_GEMM_EPI(BT)                                                                         \
    switch (epi) {                                                                                \
        case kEpiNone: return launch_bt<BT, kEpiNone>(a, tmX, tmW, tmY, ystore, num_sms, st);     \
        case kEpiBias: return launch_bt<BT, kEpiBias>(a, tmX, tmW, tmY, ystore, num_sms, st);     \
        case kEpiBiasGelu: return launch_bt<BT, kEpiBiasGelu>(a, tmX, tmW, tmY, ystore, num_sms, st); \
        case kEpiBiasRes: return launch_bt<BT, kEpiBiasRes>(a, tmX, tmW, tmY, ystore, num_sms, st);   \
        case kEpiNoneF32: return launch_bt<BT, kEpiNoneF32>(a, tmX, tmW, tmY, 0, num_sms, st);       \
        case kEpiResF32: return launch_bt<BT, kEpiResF32>(a, tmX, tmW, tmY, 0, num_sms, st);         \
        default: return cudaErrorInvalidValue;                                                    \
    }
    if (bt == 192) { MADI_GEMM_EPI(192) }
    MADI_GEMM_EPI(128)
#undef MADI_GEMM_EPI
}

}  // namespace madi
