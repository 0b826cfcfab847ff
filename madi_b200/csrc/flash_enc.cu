// flash_enc.cu -- encoder self-attention (bidirectional) on the 5th-generation tensor
// cores: m4_flash_enc (m4_gemm.metal:255-407) restated for sm_100a.
//
//   S = Q K^T * 0.125 (f32);  online softmax per query row: m' = max(m, max_j S),
//   alpha = exp(m - m'), P = exp(S - m') rounded to f16, l = l * alpha + sum(P unrounded),
//   O = O * alpha + P V (f32);  out = half(O / (l + 1e-6)).
//   q / k / v: f16 rows of `stride` elements, head h at columns h*64..h*64+63;
//   `chunks` independent sequences of `seq` rows each, back to back.
//
// One CTA per (two 128-query tiles A and B, head, chunk); 384 threads:
//   warp 0     TMA producer: the two Q tiles, then K / V tiles of 128 keys through a
//              3-stage ring (SWIZZLE_128B boxes [128 rows][64 dims]) shared by both;
//   warp 1     MMA issuer + TMEM owner.  Per key tile j and query tile x in (A, B):
//              once the softmax of x has read S_x(j) (s_free), S_x(j+1) = Q_x K_{j+1}^T
//              (M = 128 queries, N = 128 keys, K = 64 dims, both operands K-major in
//              shared memory); once it has published P_x(j) (p_ready), O_x += P_x(j) V_j
//              (TS form: P from TMEM as A, V an N-contiguous shared-memory B operand);
//   warps 4-7  softmax of tile A, warps 8-11 softmax of tile B (thread = query row =
//              TMEM lane): the row max over S in 32-column passes, then the
//              exponentials written as f16 pairs into the tile's P columns, O rescaled
//              in TMEM by alpha when a row maximum moved; finally O / l.
// Two softmax warpgroups keep the special-function unit and the tensor cores busy
// while the other group waits for its MMAs.  Back to back, an M = 128, K = 16
// tcgen05.mma takes N / 2 cycles for N >= 128, but one issuing thread starts them no
// faster than ~60 cycles apart, so the PV MMAs (N = 64) run at half the pipe's rate;
// one issuer per query tile measured slower all the same (the tiles' chains fall
// into step), so one thread issues for both tiles.
// TMEM columns of tile x: S [256x, 256x + 128), P [256x + 128, +64), O [256x + 192,
// +64).  P has its own columns, so S_x(j+1) can be computed while PV_x(j) still reads
// P_x(j); the softmax waits for PV_x(j) before it overwrites P_x.  Every wait is
// bounded.
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"

namespace madi {
namespace {

constexpr int kQT = 128;                 // queries per tile
constexpr int kKT = 128;                 // keys per tile
constexpr int kHD = 64;                  // head dim
constexpr int kNS = 3;                   // K / V ring stages (2 measured 16 % slower: loads waited for PV)
constexpr int kTile = kQT * kHD * 2;     // bytes of one [128][64] f16 tile
constexpr int kFaThreads = 384;
constexpr int kSmWarp0 = 4;              // warps 4..7: softmax of tile A; 8..11: tile B
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTileCols = 256;      // TMEM columns per query tile
constexpr uint32_t kPCol = 128;          // P columns within a tile's block
constexpr uint32_t kOCol = 192;          // O columns within a tile's block
constexpr float kScale = 0.125f;
constexpr float kLog2e = 1.4426950408889634f;

struct __align__(8) FaBars {
    uint64_t q_full;
    uint64_t kv_full[kNS];
    uint64_t kv_empty[kNS];
    uint64_t s_full[2];     // per query tile: S_x(j) computed
    uint64_t s_free[2];     // per query tile: S_x(j) read by the softmax (128 arrivals)
    uint64_t p_ready[2];    // per query tile: P_x(j) written, O_x rescaled (128 arrivals)
    uint64_t o_done[2];     // per query tile: PV_x(j) complete
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

// Two Q tiles and the K / V ring; more than half of the SM's shared memory, so a
// second CTA (which would wait in tcgen05.alloc for the 512 TMEM columns) never lands.
constexpr size_t kFaSmemUsed = 1024 + (size_t)(2 + 2 * kNS) * kTile + sizeof(FaBars) + 64;
constexpr size_t kFaSmem = kFaSmemUsed > 120 * 1024 ? kFaSmemUsed : 120 * 1024;

// PV: A = P (TMEM, K-major), B = V (shared memory, N-contiguous: bit 16 transposes B).
constexpr uint32_t kIdescS = idesc_f16_f32(kQT, kKT);
constexpr uint32_t kIdescPV = idesc_f16_f32(kQT, kHD) | (1u << 16);

// Bounded wait that ignores the abort flag (to drain work in flight before exit).
MADI_DEV void mbar_wait_drain_fa(uint64_t *bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitBudgetCycles) return;
}

// max(a, b, c) in one instruction (exact, like fmaxf on finite values).
MADI_DEV float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
MADI_DEV void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
MADI_DEV void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__global__ void __launch_bounds__(kFaThreads, 1)
    flash_enc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, __half *__restrict__ out, int out_stride, int seq,
                     int *dev_err) {
    extern __shared__ uint8_t fa_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *qs = smem;                          // 2 tiles: A, B
    uint8_t *ks = qs + 2 * kTile;                // kNS tiles
    uint8_t *vs = ks + kNS * kTile;              // kNS tiles
    FaBars *bars = reinterpret_cast<FaBars *>(vs + kNS * kTile);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * 2 * kQT, h = blockIdx.y, chunk = blockIdx.z;
    const int row0 = chunk * seq;                // first row of this chunk
    const int nkv = (seq + kKT - 1) / kKT;

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        for (int s = 0; s < kNS; ++s) {
            mbar_init(&bars->kv_full[s], 1);
            mbar_init(&bars->kv_empty[s], 1);
        }
        for (int x = 0; x < 2; ++x) {
            mbar_init(&bars->s_full[x], 1);
            mbar_init(&bars->s_free[x], 128);
            mbar_init(&bars->p_ready[x], 128);
            mbar_init(&bars->o_done[x], 1);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    volatile int *abort_flag = &bars->abort;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            // tile B may lie past the chunk (its rows are then the next chunk's, or past
            // the tensor and zero-filled); its outputs are not stored
            mbar_arrive_expect_tx(&bars->q_full, 2 * kTile);
            tma_load_2d(qs, &tmQ, &bars->q_full, h * kHD, row0 + q0);
            tma_load_2d(qs + kTile, &tmQ, &bars->q_full, h * kHD, row0 + q0 + kQT);
            int issued = 0;
            for (int j = 0; j < nkv; ++j) {
                const int s = j % kNS;
                if (!mbar_wait(&bars->kv_empty[s], ((j / kNS) & 1) ^ 1, abort_flag, dev_err)) break;
                mbar_arrive_expect_tx(&bars->kv_full[s], 2 * kTile);
                tma_load_2d(ks + s * kTile, &tmK, &bars->kv_full[s], h * kHD, row0 + j * kKT);
                tma_load_2d(vs + s * kTile, &tmV, &bars->kv_full[s], h * kHD, row0 + j * kKT);
                issued = j + 1;
            }
            // copies issued last must land before shared memory is released
            mbar_wait_drain_fa(&bars->q_full, 0);
            for (int j = issued > kNS ? issued - kNS : 0; j < issued; ++j)
                mbar_wait_drain_fa(&bars->kv_full[j % kNS], (j / kNS) & 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint64_t qd = smem_desc_sw128(smem_u32(qs));
            const uint64_t kd0 = smem_desc_sw128(smem_u32(ks));
            const uint64_t vd0 = smem_desc_sw128(smem_u32(vs));
            constexpr uint64_t kTileU = kTile >> 4;          // descriptor units per tile
            bool ok = mbar_wait(&bars->q_full, 0, abort_flag, dev_err);
            // S_x(j) = Q_x K_j^T; the K / V stage of tile j is waited for before S_A(j)
            auto issue_s = [&](int x, int j) -> bool {
                const int s = j % kNS;
                if (x == 0 && !mbar_wait(&bars->kv_full[s], (j / kNS) & 1, abort_flag, dev_err)) return false;
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < kHD / 16; ++k)       // K = 64 dims: 4 MMAs, descriptors +32 bytes each
                    mma_ss(tmem + x * kTileCols, qd + x * kTileU + 2 * k, kd0 + s * kTileU + 2 * k, kIdescS, k != 0);
                umma_commit(&bars->s_full[x]);
                return true;
            };
            if (ok) ok = issue_s(0, 0) && issue_s(1, 0);
            for (int j = 0; ok && j < nkv; ++j) {
                const int s = j % kNS;
                for (int x = 0; ok && x < 2; ++x) {
                    // the next S as soon as the softmax has read S_x(j) (it still computes
                    // the last exponentials and the rescale), then PV_x(j) once P_x(j) is out
                    if (j + 1 < nkv) {
                        if (!mbar_wait(&bars->s_free[x], j & 1, abort_flag, dev_err) || !issue_s(x, j + 1)) {
                            ok = false;
                            break;
                        }
                    }
                    if (!mbar_wait(&bars->p_ready[x], j & 1, abort_flag, dev_err)) { ok = false; break; }
                    tc_fence_after();
                    // O_x += P_x(j) V_j: K = 128 keys in 8 steps; P columns +8 (16 f16), V rows +16 = 2048 bytes
                    const uint32_t tb = tmem + x * kTileCols;
#pragma unroll
                    for (int k = 0; k < kKT / 16; ++k)
                        mma_ts(tb + kOCol, tb + kPCol + 8 * k, vd0 + s * kTileU + 128 * k, kIdescPV, (j | k) != 0);
                    umma_commit(&bars->o_done[x]);
                }
                if (ok) umma_commit(&bars->kv_empty[s]);
            }
            umma_commit(&bars->drain);
            mbar_wait_drain_fa(&bars->drain, 0);
        }
        __syncwarp();
    } else if (warp >= kSmWarp0) {
        // ------------------------------------------------ softmax, one query row per thread
        const int x = (warp - kSmWarp0) >> 2;      // query tile of this warpgroup
        const int qw = warp & 3;
        const uint32_t lane_addr = (uint32_t)(qw * 32) << 16;
        const uint32_t tb = tmem + lane_addr + x * kTileCols;
        const int qrow = qw * 32 + lane;         // row of the tile
        float m = -INFINITY, l = 0.f;
        bool alive = true;
        for (int j = 0; j < nkv && alive; ++j) {
            alive = warp_wait_all(&bars->s_full[x], j & 1, abort_flag, dev_err);
            if (!alive) break;
            tc_fence_after();
            const int kcur = min(seq - j * kKT, kKT);   // valid keys of this tile
            const bool full = kcur == kKT;
            // row max of the raw scores (scale > 0 commutes with max), 32 columns per
            // pass; keys >= kcur masked.  A full tile (every tile but a chunk's last)
            // keeps eight partial maxima (max is exact in any order) and no per-key mask.
            // Loads run one chunk ahead of the arithmetic (tcgen05.wait::ld waits for all
            // of this thread's loads, so chunk c + 1 is in flight while chunk c is used).
            float mx[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
            uint32_t sv[2][32];
            tmem_ld32(tb, sv[0]);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < kKT / 32; ++c) {
                if (c + 1 < kKT / 32) tmem_ld32(tb + 32 * (c + 1), sv[(c + 1) & 1]);
                const uint32_t (&cv)[32] = sv[c & 1];
                if (full) {
#pragma unroll
                    for (int i = 0; i < 32; i += 2)    // three-input max: two scores per instruction
                        mx[(i >> 1) & 7] = max3f(mx[(i >> 1) & 7], __uint_as_float(cv[i]), __uint_as_float(cv[i + 1]));
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (32 * c + i < kcur) mx[i & 7] = fmaxf(mx[i & 7], __uint_as_float(cv[i]));
                }
                if (c + 1 < kKT / 32) tmem_wait_ld();
            }
            const float mxr =
                fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
            const float mn = fmaxf(m, mxr * kScale);
            // exp(s * scale - m') = 2^(s * scale * log2 e - m' * log2 e): one FFMA and the
            // hardware base-2 exponential per element (P is rounded to f16 after it)
            const float ml = mn * kLog2e;
            // exactly 1 when the row max did not move: the O rescale below runs when any
            // row of the warp grew (rows past the chunk end included), and it must then
            // leave the other rows' O bit-for-bit unchanged
            const float alpha = (m == -INFINITY) ? 0.f : (mn == m ? 1.f : ex2_approx(fmaf(m, kLog2e, -ml)));
            // P_x(j - 1) must have been read by PV_x(j - 1) before P_x(j) overwrites it;
            // that also makes O_x complete for the rescale below
            if (j > 0) {
                alive = warp_wait_all(&bars->o_done[x], (j - 1) & 1, abort_flag, dev_err);
                if (!alive) break;
                tc_fence_after();
            }
            // row sum of the unrounded P over eight partial sums (even and odd keys of four
            // interleaved groups: shorter dependency chains, packed adds)
            float bq[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            tmem_ld32(tb, sv[0]);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < kKT / 32; ++c) {
                if (c + 1 < kKT / 32) tmem_ld32(tb + 32 * (c + 1), sv[(c + 1) & 1]);
                const uint32_t (&cv)[32] = sv[c & 1];
                uint32_t pp[16];
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const int key = 32 * c + i;
                    const int g = (i >> 1) & 3;
                    float e0, e1;
                    if (full) {
                        // both exponents in one packed FMA (each lane rounded as fmaf)
                        float a0, a1;
                        fma2(a0, a1, __uint_as_float(cv[i]), __uint_as_float(cv[i + 1]), kScale * kLog2e,
                             kScale * kLog2e, -ml, -ml);
                        e0 = ex2_approx(a0);
                        e1 = ex2_approx(a1);
                    } else {
                        e0 = key < kcur ? ex2_approx(fmaf(__uint_as_float(cv[i]), kScale * kLog2e, -ml)) : 0.f;
                        e1 = key + 1 < kcur ? ex2_approx(fmaf(__uint_as_float(cv[i + 1]), kScale * kLog2e, -ml)) : 0.f;
                    }
                    add2(bq[2 * g], bq[2 * g + 1], bq[2 * g], bq[2 * g + 1], e0, e1);
                    pp[i >> 1] = h2_as_u32(__floats2half2_rn(e0, e1));
                }
                tmem_st16(tb + kPCol + 16 * c, pp);
                if (c + 1 < kKT / 32) {
                    tmem_wait_ld();
                    if (c + 2 == kKT / 32) {
                        // the last chunk of S_x(j) is in registers: the MMA thread may
                        // overwrite S_x with S_x(j + 1)
                        tc_fence_before();
                        mbar_arrive(&bars->s_free[x]);
                    }
                }
            }
            const float bs = ((bq[0] + bq[1]) + (bq[2] + bq[3])) + ((bq[4] + bq[5]) + (bq[6] + bq[7]));
            l = l * alpha + bs;
            const bool grew = mn != m;
            m = mn;
            if (j > 0 && __any_sync(0xffffffffu, grew)) {
                // O *= alpha; skipped when no row of the warp has a new maximum
                uint32_t ov[32];
#pragma unroll
                for (int c = 0; c < kHD / 32; ++c) {
                    tmem_ld32(tb + kOCol + 32 * c, ov);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        float o0, o1;
                        mul2(o0, o1, __uint_as_float(ov[i]), __uint_as_float(ov[i + 1]), alpha, alpha);
                        ov[i] = __float_as_uint(o0);
                        ov[i + 1] = __float_as_uint(o1);
                    }
                    tmem_st32(tb + kOCol + 32 * c, ov);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars->p_ready[x]);
        }
        if (alive) alive = warp_wait_all(&bars->o_done[x], (nkv - 1) & 1, abort_flag, dev_err);
        if (alive) {
            tc_fence_after();
            const int q = q0 + x * kQT + qrow;
            const float inv = 1.0f / (l + 1e-6f);
            __half *orow = out + (size_t)(row0 + q) * out_stride + h * kHD;
#pragma unroll
            for (int c = 0; c < kHD / 32; ++c) {
                uint32_t ov[32];
                tmem_ld32(tb + kOCol + 32 * c, ov);
                tmem_wait_ld();
                if (q < seq) {
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        uint4 w;
                        w.x = h2_as_u32(__floats2half2_rn(__uint_as_float(ov[8 * g]) * inv, __uint_as_float(ov[8 * g + 1]) * inv));
                        w.y = h2_as_u32(__floats2half2_rn(__uint_as_float(ov[8 * g + 2]) * inv, __uint_as_float(ov[8 * g + 3]) * inv));
                        w.z = h2_as_u32(__floats2half2_rn(__uint_as_float(ov[8 * g + 4]) * inv, __uint_as_float(ov[8 * g + 5]) * inv));
                        w.w = h2_as_u32(__floats2half2_rn(__uint_as_float(ov[8 * g + 6]) * inv, __uint_as_float(ov[8 * g + 7]) * inv));
                        *reinterpret_cast<uint4 *>(orow + 32 * c + 8 * g) = w;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

bool fa_map(CUtensorMap *m, const void *base, uint64_t rows, int stride, int cols) {
    PFN_encodeTiled enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, rows};
    const cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kHD, (cuuint32_t)kQT};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_flash_enc(const __half *q, const __half *k, const __half *v, int stride, __half *out,
                             int out_stride, int seq, int heads, int chunks, int *dev_err, cudaStream_t st) {
    CUtensorMap tmQ, tmK, tmV;
    const uint64_t rows = (uint64_t)chunks * seq;
    const int cols = heads * kHD;
    if (!fa_map(&tmQ, q, rows, stride, cols) || !fa_map(&tmK, k, rows, stride, cols) ||
        !fa_map(&tmV, v, rows, stride, cols))
        return cudaErrorNotSupported;
    static std::once_flag once;
    static cudaError_t once_status;
    if (cudaError_t e = run_once(once, once_status, [] {
            return cudaFuncSetAttribute(flash_enc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFaSmem);
        }))
        return e;
    const dim3 grid((seq + 2 * kQT - 1) / (2 * kQT), heads, chunks);
    flash_enc_kernel<<<grid, kFaThreads, kFaSmem, st>>>(tmQ, tmK, tmV, out, out_stride, seq, dev_err);
    return cudaGetLastError();
}

}  // namespace madi
