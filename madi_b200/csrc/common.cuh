// common.cuh -- device helpers shared by the sm_100a Q8 kernels.
//
//  * exact int8 -> f16 conversion (bias-exponent trick, see q8_to_half2x2)
//  * Abramowitz & Stegun 7.1.26 GELU, the reference's epilogue formula
//    (m4_gemm.metal:43-57, graph_helpers.metal:460-473)
//  * thin inline-PTX wrappers: mbarrier, TMA (cp.async.bulk.tensor), tcgen05
//  * bounded waits: every spin has a clock budget; on expiry it raises the
//    CTA's abort flag and the library's device error word instead of hanging.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define MADI_DEV __device__ __forceinline__

namespace madi {

// ~2 s at 1.9 GHz: far above any legitimate wait in these kernels.
constexpr long long kWaitBudgetCycles = 4000000000LL;

// Device error word codes (written with atomicCAS so the first cause sticks).
enum : int { kDevErrNone = 0, kDevErrWaitTimeout = 1, kDevErrBadArgs = 2 };

// ------------------------------------------------------------------ numerics

// Four int8 (one 32-bit word, little-endian) -> two half2 holding q exactly:
// lo = {q0, q1}, hi = {q2, q3}.  Flipping the sign bit turns q into the
// unsigned byte q+128; placing that byte under the f16 exponent of 1024
// (0x64xx) gives the half 1024 + q + 128 exactly; subtracting 1152 leaves q.
MADI_DEV void q8_to_half2x2(uint32_t w, __half2 &lo, __half2 &hi) {
    const uint32_t u = w ^ 0x80808080u;
    uint32_t a, b;
    asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(a) : "r"(u), "r"(0x64646464u));
    asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(b) : "r"(u), "r"(0x64646464u));
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    lo = __hsub2(*reinterpret_cast<__half2 *>(&a), bias);
    hi = __hsub2(*reinterpret_cast<__half2 *>(&b), bias);
}

MADI_DEV uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// ------------------------------------------------------ programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while the
// kernel before it still runs.  pdl_wait() blocks until that kernel has finished
// and its writes are visible (a no-op without the launch attribute); every kernel
// launched that way calls it on every path before reading data another kernel
// wrote and before it can finish, so completion stays ordered along the stream.
// pdl_trigger() lets the next kernel of the stream start launching.
MADI_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MADI_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// 0.5 x (1 + erf(x / sqrt 2)), erf from A&S 7.1.26 (|eps| <= 1.5e-7) with
// exp2(max(-z^2 log2 e, -80)): the reference's GELU formula, restated.
// Written as 0.5 x + 0.5 |x| erf(|z|) (erf is odd, so sign(x) x = |x|).  The
// reciprocal and exp2 are the single hardware approximations (rcp.approx,
// ex2.approx); their error is far below the 2e-3 x RMS output tolerance.
MADI_DEV float rcp_approx(float v) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}
MADI_DEV float ex2_approx(float v) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}
MADI_DEV float gelu_erf(float xv) {
    const float az = fabsf(xv) * 0.7071067811865476f;
    const float t = rcp_approx(fmaf(az, 0.3275911f, 1.0f));
    float poly = fmaf(1.061405429f, t, -1.453152027f);
    poly = fmaf(poly, t, 1.421413741f);
    poly = fmaf(poly, t, -0.284496736f);
    poly = fmaf(poly, t, 0.254829592f);
    poly = poly * t;
    const float ex = ex2_approx(fmaxf(az * az * -1.4426950408889634f, -80.0f));
    const float erf_abs = fmaf(-poly, ex, 1.0f);
    const float h = 0.5f * xv;
    return fmaf(fabsf(h), erf_abs, h);
}

// Packed f32x2 arithmetic (sm_100): two IEEE f32 operations per instruction,
// each lane rounded exactly as the scalar operation.
MADI_DEV void fma2(float &d0, float &d1, float a0, float a1, float b0, float b1, float c0, float c1) {
    asm("{\n\t.reg .b64 a, b, c, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
        "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
MADI_DEV void mul2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "mul.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
MADI_DEV void add2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "add.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// gelu_erf of two values with packed arithmetic, bit-identical to gelu_erf on
// each: the same operations in the same order.  The polynomial runs on negated
// coefficients, giving -poly exactly (round-to-nearest is symmetric), so
// 1 - poly * ex is one FMA without a separate negation.
MADI_DEV void gelu_erf2(float &y0, float &y1, float x0, float x1) {
    float az0, az1, d0, d1, np0, np1, s0, s1, e0, e1, h0, h1;
    mul2(az0, az1, fabsf(x0), fabsf(x1), 0.7071067811865476f, 0.7071067811865476f);
    fma2(d0, d1, az0, az1, 0.3275911f, 0.3275911f, 1.0f, 1.0f);
    const float t0 = rcp_approx(d0), t1 = rcp_approx(d1);
    fma2(np0, np1, -1.061405429f, -1.061405429f, t0, t1, 1.453152027f, 1.453152027f);
    fma2(np0, np1, np0, np1, t0, t1, -1.421413741f, -1.421413741f);
    fma2(np0, np1, np0, np1, t0, t1, 0.284496736f, 0.284496736f);
    fma2(np0, np1, np0, np1, t0, t1, -0.254829592f, -0.254829592f);
    mul2(np0, np1, np0, np1, t0, t1);
    mul2(s0, s1, az0, az1, az0, az1);
    mul2(s0, s1, s0, s1, -1.4426950408889634f, -1.4426950408889634f);
    const float ex0 = ex2_approx(fmaxf(s0, -80.0f)), ex1 = ex2_approx(fmaxf(s1, -80.0f));
    fma2(e0, e1, np0, np1, ex0, ex1, 1.0f, 1.0f);
    mul2(h0, h1, 0.5f, 0.5f, x0, x1);
    fma2(y0, y1, fabsf(h0), fabsf(h1), e0, e1, h0, h1);
}

// ------------------------------------------------------------------ shared / mbarrier

MADI_DEV uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

MADI_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
MADI_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

MADI_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}
MADI_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
// A waiting thread may sleep up to kSuspendNs inside one try_wait (it wakes when the
// phase completes), so a warp that waits does not keep issuing polling
// instructions beside the warps that work; the callers' abort-flag and clock-budget
// checks still run at least this often.
constexpr uint32_t kSuspendNs = 1000000;
MADI_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// Waits for `parity` on `bar`.  Gives up (returns false) when the CTA abort
// flag is raised or the clock budget runs out; in the latter case it raises
// the abort flag and records kDevErrWaitTimeout in *dev_err.
MADI_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *dev_err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitBudgetCycles) {
            *abort_flag = 1;
            if (dev_err) atomicCAS(dev_err, kDevErrNone, kDevErrWaitTimeout);
            return false;
        }
    }
}

// Warp-uniform bounded wait: every lane observes the barrier (so each has the
// acquire ordering for the data it guards), then the warp agrees; a lane that
// gave up makes the whole warp give up, keeping warp-collective ops convergent.
MADI_DEV bool warp_wait_all(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *dev_err) {
    const bool ok = mbar_wait(bar, parity, abort_flag, dev_err);
    return __all_sync(0xffffffffu, ok);
}

// ------------------------------------------------------------------ prefetching loads

// Read-only predicated loads into a register the caller pre-set (kept when the
// predicate is false).  Nothing consumes the value inside the asm, so the
// thread only waits for it at its first real use: a register prefetch.
MADI_DEV void ldg_nc_u32_pred(uint32_t &dst, const void *p, bool pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q ld.global.nc.b32 %0, [%1];\n\t}"
                 : "+r"(dst)
                 : "l"(p), "r"((int)pred));
}
MADI_DEV void ldg_nc_u16_pred(uint32_t &dst, const void *p, bool pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q ld.global.nc.u16 %0, [%1];\n\t}"
                 : "+r"(dst)
                 : "l"(p), "r"((int)pred));
}

// ------------------------------------------------------------------ TMA

MADI_DEV void tma_prefetch_desc(const CUtensorMap *m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 2-D tiled TMA load (no multicast) into this CTA's shared memory; completes
// `bytes` of transaction on `bar`.  c0 = innermost coordinate (elements).
MADI_DEV void tma_load_2d(void *smem_dst, const CUtensorMap *m, uint64_t *bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// 3-D tiled TMA load (no multicast); c0 = innermost coordinate (elements).
MADI_DEV void tma_load_3d(void *smem_dst, const CUtensorMap *m, uint64_t *bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// 2-D tiled TMA store shared::cta -> global (bulk-group completion); the tensor
// map clips rows and columns outside the tensor.  c0 = innermost coordinate.
MADI_DEV void tma_store_2d(const CUtensorMap *m, const void *smem_src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
                 : "memory");
}
MADI_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups still read their shared-memory source.
template <int N> MADI_DEV void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
MADI_DEV void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Generic-proxy shared-memory writes before this fence are visible to later
// async-proxy (TMA) reads once a barrier orders them.
MADI_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
MADI_DEV void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------ tcgen05

MADI_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MADI_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Warp-collective.  Writes the TMEM base address to *dst_smem.
MADI_DEV void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
MADI_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
MADI_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]; kind::f16, single CTA.  One thread issues.
MADI_DEV void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// One 64-wide K stage of a TS MMA chain in a single asm block: four K=16 MMAs
// (A columns advance by 8, the B descriptor's start address by 32 bytes = 2 in
// its 16-byte units) followed by two commits.  `desc_lo`/`desc_hi` are the two
// words of the K-major SWIZZLE_128B smem descriptor of the stage's first MMA;
// `accumulate` = 0 starts a new accumulation with the first MMA.
MADI_DEV void umma_stage4_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t desc_lo, uint32_t desc_hi, uint32_t idesc,
                             uint32_t accumulate, uint32_t bar0, uint32_t bar1) {
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b32 a1, a2, a3, l1, l2, l3;\n\t.reg .b64 d0, d1, d2, d3;\n\t"
        "setp.ne.b32 p, %4, 0;\n\tsetp.eq.b32 t, %4, %4;\n\t"
        "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
        "add.u32 l1, %2, 2;\n\tadd.u32 l2, %2, 4;\n\tadd.u32 l3, %2, 6;\n\t"
        "mov.b64 d0, {%2, %3};\n\tmov.b64 d1, {l1, %3};\n\tmov.b64 d2, {l2, %3};\n\tmov.b64 d3, {l3, %3};\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], d0, %5, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], d1, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], d2, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], d3, %5, t;\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "r"(desc_lo), "r"(desc_hi), "r"(accumulate), "r"(idesc), "r"(bar0), "r"(bar1)
        : "memory");
}

// Two consecutive 64-wide K stages in one asm block: the second stage's A
// columns follow the first's (+32) and its B tile is `desc_step` 16-byte units
// further; eight MMAs, then four commits (bar0..bar3).
MADI_DEV void umma_stage8_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t desc_lo, uint32_t desc_hi, uint32_t desc_step,
                             uint32_t idesc, uint32_t accumulate, uint32_t bar0, uint32_t bar1, uint32_t bar2,
                             uint32_t bar3) {
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b32 a1, a2, a3, a4, a5, a6, a7, l1, l2, l3, l4, l5, l6, l7;\n\t"
        ".reg .b64 d0, d1, d2, d3, d4, d5, d6, d7;\n\t"
        "setp.ne.b32 p, %4, 0;\n\tsetp.eq.b32 t, %4, %4;\n\t"
        "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
        "add.u32 a4, %1, 32;\n\tadd.u32 a5, %1, 40;\n\tadd.u32 a6, %1, 48;\n\tadd.u32 a7, %1, 56;\n\t"
        "add.u32 l1, %2, 2;\n\tadd.u32 l2, %2, 4;\n\tadd.u32 l3, %2, 6;\n\t"
        "add.u32 l4, %2, %6;\n\tadd.u32 l5, l4, 2;\n\tadd.u32 l6, l4, 4;\n\tadd.u32 l7, l4, 6;\n\t"
        "mov.b64 d0, {%2, %3};\n\tmov.b64 d1, {l1, %3};\n\tmov.b64 d2, {l2, %3};\n\tmov.b64 d3, {l3, %3};\n\t"
        "mov.b64 d4, {l4, %3};\n\tmov.b64 d5, {l5, %3};\n\tmov.b64 d6, {l6, %3};\n\tmov.b64 d7, {l7, %3};\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], d0, %5, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], d1, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], d2, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], d3, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a4], d4, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a5], d5, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a6], d6, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a7], d7, %5, t;\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%8];\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%9];\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%10];\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "r"(desc_lo), "r"(desc_hi), "r"(accumulate), "r"(idesc), "r"(desc_step), "r"(bar0), "r"(bar1),
        "r"(bar2), "r"(bar3)
        : "memory");
}

// As umma_stage8_ts with two commits (both stages' resources released through
// one barrier each).
MADI_DEV void umma_stage8_ts_2c(uint32_t d_tmem, uint32_t a_tmem, uint32_t desc_lo, uint32_t desc_hi,
                                uint32_t desc_step, uint32_t idesc, uint32_t accumulate, uint32_t bar0, uint32_t bar1) {
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b32 a1, a2, a3, a4, a5, a6, a7, l1, l2, l3, l4, l5, l6, l7;\n\t"
        ".reg .b64 d0, d1, d2, d3, d4, d5, d6, d7;\n\t"
        "setp.ne.b32 p, %4, 0;\n\tsetp.eq.b32 t, %4, %4;\n\t"
        "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
        "add.u32 a4, %1, 32;\n\tadd.u32 a5, %1, 40;\n\tadd.u32 a6, %1, 48;\n\tadd.u32 a7, %1, 56;\n\t"
        "add.u32 l1, %2, 2;\n\tadd.u32 l2, %2, 4;\n\tadd.u32 l3, %2, 6;\n\t"
        "add.u32 l4, %2, %6;\n\tadd.u32 l5, l4, 2;\n\tadd.u32 l6, l4, 4;\n\tadd.u32 l7, l4, 6;\n\t"
        "mov.b64 d0, {%2, %3};\n\tmov.b64 d1, {l1, %3};\n\tmov.b64 d2, {l2, %3};\n\tmov.b64 d3, {l3, %3};\n\t"
        "mov.b64 d4, {l4, %3};\n\tmov.b64 d5, {l5, %3};\n\tmov.b64 d6, {l6, %3};\n\tmov.b64 d7, {l7, %3};\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], d0, %5, p;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], d1, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], d2, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], d3, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a4], d4, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a5], d5, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a6], d6, %5, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a7], d7, %5, t;\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n\t"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%8];\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "r"(desc_lo), "r"(desc_hi), "r"(accumulate), "r"(idesc), "r"(desc_step), "r"(bar0), "r"(bar1)
        : "memory");
}

// ------------------------------------------------------------------ CTA pairs (cta_group::2)
//
// A cluster of two CTAs on neighbouring SMs shares each MMA: the even CTA's
// thread issues tcgen05.mma.cta_group::2 with M = 256; rows 0-127 of A and D
// live in the even CTA's tensor memory, rows 128-255 in the odd CTA's, and B's
// N columns are the two CTAs' shared-memory tiles side by side (first half in
// the even CTA).  Every tcgen05 instruction that names a CTA group uses ::2.

MADI_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// All threads of both CTAs; orders shared-memory state across the pair.
MADI_DEV void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
MADI_DEV uint32_t mapa_u32(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Arrive on the barrier at cluster address `cbar` (possibly in the peer CTA),
// with the instruction's default semantics (release at CTA scope).  The data
// these arrivals publish lives in tensor memory and is ordered by the
// tcgen05.fence::before_thread_sync / after_thread_sync pair around them; a
// cluster-scope release would add a cluster-wide fence to every arrival.
MADI_DEV void mbar_arrive_cluster(uint32_t cbar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cbar) : "memory");
}
MADI_DEV void st_cluster_u32(uint32_t caddr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(caddr), "r"(v) : "memory");
}
// mbar_wait for CTA pairs: on budget expiry it raises this CTA's abort flag and
// the peer's (cluster address `peer_abort`), so both stop promptly.  Waits are
// at CTA scope, as the arrivals they pair with (see mbar_arrive_cluster).
MADI_DEV bool mbar_wait_cl(uint64_t *bar, uint32_t parity, volatile int *abort_flag, uint32_t peer_abort,
                           int *dev_err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitBudgetCycles) {
            *abort_flag = 1;
            st_cluster_u32(peer_abort, 1u);
            if (dev_err) atomicCAS(dev_err, kDevErrNone, kDevErrWaitTimeout);
            return false;
        }
    }
}
MADI_DEV bool warp_wait_all_cl(uint64_t *bar, uint32_t parity, volatile int *abort_flag, uint32_t peer_abort,
                               int *dev_err) {
    const bool ok = mbar_wait_cl(bar, parity, abort_flag, peer_abort, dev_err);
    return __all_sync(0xffffffffu, ok);
}

// Warp-collective, executed by the same warp in both CTAs of the pair.
MADI_DEV void tmem_alloc2(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
MADI_DEV void tmem_relinquish2() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
MADI_DEV void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Arrive on `bar` in both CTAs of the pair once the pair's tcgen05 ops issued so
// far by this thread complete.
MADI_DEV void umma2_commit_both(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}

// Pair form of umma_stage4_ts: four K=16 MMAs of M = 256, then two commits, each
// arriving on its barrier in both CTAs.
MADI_DEV void umma2_stage4_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t desc_lo, uint32_t desc_hi, uint32_t idesc,
                              uint32_t accumulate, uint32_t bar0, uint32_t bar1) {
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b32 a1, a2, a3, l1, l2, l3;\n\t.reg .b64 d0, d1, d2, d3;\n\t"
        "setp.ne.b32 p, %4, 0;\n\tsetp.eq.b32 t, %4, %4;\n\t"
        "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
        "add.u32 l1, %2, 2;\n\tadd.u32 l2, %2, 4;\n\tadd.u32 l3, %2, 6;\n\t"
        "mov.b64 d0, {%2, %3};\n\tmov.b64 d1, {l1, %3};\n\tmov.b64 d2, {l2, %3};\n\tmov.b64 d3, {l3, %3};\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], d0, %5, p;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a1], d1, %5, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a2], d2, %5, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a3], d3, %5, t;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%6], %8;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%7], %8;\n\t}" ::"r"(
            d_tmem),
        "r"(a_tmem), "r"(desc_lo), "r"(desc_hi), "r"(accumulate), "r"(idesc), "r"(bar0), "r"(bar1),
        "h"((uint16_t)3)
        : "memory");
}

// Pair form of umma_stage8_ts_2c: two consecutive K stages (eight MMAs of M = 256),
// then two commits arriving in both CTAs.
MADI_DEV void umma2_stage8_ts_2c(uint32_t d_tmem, uint32_t a_tmem, uint32_t desc_lo, uint32_t desc_hi,
                                 uint32_t desc_step, uint32_t idesc, uint32_t accumulate, uint32_t bar0,
                                 uint32_t bar1) {
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b32 a1, a2, a3, a4, a5, a6, a7, l1, l2, l3, l4, l5, l6, l7;\n\t"
        ".reg .b64 d0, d1, d2, d3, d4, d5, d6, d7;\n\t"
        "setp.ne.b32 p, %4, 0;\n\tsetp.eq.b32 t, %4, %4;\n\t"
        "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
        "add.u32 a4, %1, 32;\n\tadd.u32 a5, %1, 40;\n\tadd.u32 a6, %1, 48;\n\tadd.u32 a7, %1, 56;\n\t"
        "add.u32 l1, %2, 2;\n\tadd.u32 l2, %2, 4;\n\tadd.u32 l3, %2, 6;\n\t"
        "add.u32 l4, %2, %6;\n\tadd.u32 l5, l4, 2;\n\tadd.u32 l6, l4, 4;\n\tadd.u32 l7, l4, 6;\n\t"
        "mov.b64 d0, {%2, %3};\n\tmov.b64 d1, {l1, %3};\n\tmov.b64 d2, {l2, %3};\n\tmov.b64 d3, {l3, %3};\n\t"
        "mov.b64 d4, {l4, %3};\n\tmov.b64 d5, {l5, %3};\n\tmov.b64 d6, {l6, %3};\n\tmov.b64 d7, {l7, %3};\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], d0, %5, p;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a1], d1, %5, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a2], d2, %5, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a3], d3, %5, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a4], d4, %5, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a5], d5, %5, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a6], d6, %5, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a7], d7, %5, t;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%7], %9;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%8], %9;\n\t}" ::"r"(
            d_tmem),
        "r"(a_tmem), "r"(desc_lo), "r"(desc_hi), "r"(accumulate), "r"(idesc), "r"(desc_step), "r"(bar0), "r"(bar1),
        "h"((uint16_t)3)
        : "memory");
}

// Arrive on `bar` once every tcgen05 op issued so far by this thread completes.
MADI_DEV void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

MADI_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
MADI_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns (thread = lane, register i = column i).
MADI_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

MADI_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),
        "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns.
MADI_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte swizzle layout that TMA's SWIZZLE_128B writes: rows of 128 bytes,
// 8-row groups 1024 bytes apart (SBO), LBO unused (1), descriptor version 1.
MADI_DEV uint64_t smem_desc_sw128(uint32_t smem_addr) {
    return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: A = B = f16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

}  // namespace madi
