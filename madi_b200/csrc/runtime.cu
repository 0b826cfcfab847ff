// runtime.cu -- the C ABI declared in include/madi_q8.h.
//
// Re-expresses the reference's Metal bridge (engine/metal/metal_backend.m) for
// CUDA on B200:
//   mtl_init / cleanup            -> device bind, library stream, sm_100 check
//   mtl_alloc registry (:136-230) -> cudaMalloc + an ordered registry so base
//                                    and interior pointers resolve (:756-790)
//   mtl_get_function (:607-666)   -> name table of the reference Q8 kernels
//   mtl_dispatch (:669-797)       -> argument unpacking in kernelParams style,
//                                    validation, B200 launch (own grid/block)
//   command buffers (:861-917)    -> CUDA stream capture -> CUDA graph replay
//   mtl_sync (:816-859)           -> bounded event poll (+ device error word)
//   per-kernel profiler (:107-132, :717-747) -> CUDA events, kern_sum table
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/madi_q8.h"
#include "internal.h"

namespace {

using namespace madi;

thread_local std::string g_last_error = "ok";

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}
int cuda_fail(cudaError_t e, const char *what) {
    return fail(MADI_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

struct State {
    bool ready = false;
    int device = -1;
    int num_sms = 0;
    int max_smem_optin = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;   // current (own or caller's)
    int *dev_err = nullptr;          // device error word (bounded-wait expiry)
    bool capturing = false;
    cudaGraphExec_t exec = nullptr;
    cudaEvent_t done = nullptr;
    int verbose = 0;
    bool profile = false;
    bool pdl = true;
    std::map<std::string, std::pair<long long, double>> prof;   // name -> (instances, total ms)
} S;

}  // namespace

namespace madi {
bool pdl_on() { return S.pdl; }
int num_sms() { return S.num_sms > 0 ? S.num_sms : 148; }
}  // namespace madi

namespace {

std::mutex g_alloc_mu;
std::map<uintptr_t, size_t> g_allocs;   // base -> size

bool in_registry(const void *p) {
    std::lock_guard<std::mutex> lk(g_alloc_mu);
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    auto it = g_allocs.upper_bound(a);
    if (it == g_allocs.begin()) return false;
    --it;
    return a < it->first + it->second;
}

bool is_device_ptr(const void *p) {
    if (!p) return false;
    if (in_registry(p)) return true;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Bytes from p to the end of the device allocation that contains it (0 if
// unknown): the bound for indices the by-name decode-step kernels read from
// device memory (positions, tokens), whose reference signatures carry no
// buffer lengths.
size_t bytes_after(const void *p) {
    typedef CUresult (*PFN_range)(CUdeviceptr *, size_t *, CUdeviceptr);
    static PFN_range fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_range>(ptr);
    });
    CUdeviceptr base = 0;
    size_t size = 0;
    if (!fn || !p || fn(&base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return 0;
    return (size_t)(base + size - reinterpret_cast<CUdeviceptr>(p));
}

cudaStream_t pick_stream(void *s) { return s ? static_cast<cudaStream_t>(s) : S.stream; }

// ---------------------------------------------------------------- Q8 linear core

int q8_linear_impl(const madi_q8w *w, const void *x, int x_dtype, int m, const void *bias, int bias_dtype, int epi,
                   const void *residual, void *y, int y_dtype, cudaStream_t st, const char *who) {
    if (!S.ready) return fail(MADI_ENOINIT, "%s: madi_init has not succeeded", who);
    if (!w || !w->qs || !w->scales) return fail(MADI_EINVAL, "%s: null weight", who);
    const int N = w->n, K = w->k;
    if (N <= 0 || K <= 0 || (K % 32) != 0) return fail(MADI_EINVAL, "%s: bad weight shape N=%d K=%d (K %% 32 == 0)", who, N, K);
    if (m <= 0) return fail(MADI_EINVAL, "%s: m=%d must be > 0", who, m);
    if (!x || !y) return fail(MADI_EINVAL, "%s: null x or y", who);
    if (epi < MADI_EPI_NONE || epi > MADI_EPI_BIAS_RES) return fail(MADI_EINVAL, "%s: bad epilogue %d", who, epi);
    if (epi != MADI_EPI_NONE && !bias) return fail(MADI_EINVAL, "%s: epilogue %d needs a bias", who, epi);
    if (epi == MADI_EPI_BIAS_RES && !residual) return fail(MADI_EINVAL, "%s: residual epilogue needs a residual", who);
    if ((x_dtype != MADI_F32 && x_dtype != MADI_F16 && x_dtype != MADI_F32_AS_F16) ||
        (y_dtype != MADI_F32 && y_dtype != MADI_F16) || (bias && bias_dtype != MADI_F32 && bias_dtype != MADI_F16))
        return fail(MADI_EINVAL, "%s: bad dtype", who);
    const bool x_r16 = x_dtype == MADI_F32_AS_F16;
    if (x_r16) x_dtype = MADI_F32;
    if ((size_t)m * (size_t)std::max(N, K) >= (1ull << 31) || (size_t)N * K >= (1ull << 40))
        return fail(MADI_EINVAL, "%s: problem too large (m=%d N=%d K=%d)", who, m, N, K);
    if (!aligned(w->qs, 16) || !aligned(w->scales, 2)) return fail(MADI_EINVAL, "%s: qs must be 16-byte aligned", who);

    // m <= 16 token rows take the streaming skinny GEMM when its tile plan fits (all
    // K % 256 == 0 shapes of the decoder and the head); larger m, or m in 9..16 with
    // another K, the tensor-core GEMM.
    const bool x_al = aligned(x, x_dtype == MADI_F32 ? 16 : 8);
    const bool tile_fits = m <= kGemvMaxM && x_al && aligned(w->scales, 16) &&
                           gemv_tile_ok(m, N, K, x_dtype == MADI_F32 && !x_r16, S.num_sms);
    if (x_r16 && !tile_fits)
        return fail(MADI_EINVAL, "%s: MADI_F32_AS_F16 activations need the streaming path (m <= %d, K %% 256 == 0, "
                                 "16-byte aligned x and scales)", who, kGemvMaxM);
    if (m >= kGemmMinM && !tile_fits) {
        const bool y32 = y_dtype == MADI_F32;
        if (x_dtype != MADI_F16 || (y32 && epi != MADI_EPI_NONE && epi != MADI_EPI_BIAS_RES))
            return fail(MADI_EINVAL, "%s: the tensor-core path (m > 8) takes f16 x, and f16 y (f32 y without an "
                                     "epilogue, or with the f32 residual stream)", who);
        if (!aligned(x, 16)) return fail(MADI_EINVAL, "%s: x must be 16-byte aligned", who);
        if (!aligned(y, y32 ? 4 : 2) || (residual && !aligned(residual, y32 ? 4 : 2)))
            return fail(MADI_EINVAL, "%s: misaligned y", who);
        GemmArgs a{};
        a.x = static_cast<const __half *>(x);
        a.qs = w->qs;
        a.scales = reinterpret_cast<const __half *>(w->scales);
        a.bias = bias;
        a.bias_f16 = bias_dtype == MADI_F16;
        a.residual = residual;
        a.y = static_cast<__half *>(y);
        a.M = m; a.N = N; a.K = K;
        a.dev_err = S.dev_err;
        cudaError_t e = launch_gemm_tc(a, y32 ? (epi == MADI_EPI_BIAS_RES ? kEpiResF32 : kEpiNoneF32) : epi, S.num_sms,
                                       st);
        if (e == cudaErrorNotSupported) return fail(MADI_EUNSUPPORTED, "%s: cuTensorMapEncodeTiled unavailable", who);
        if (e != cudaSuccess) return cuda_fail(e, who);
        return MADI_OK;
    }
    const bool xf32 = x_dtype == MADI_F32;
    if (!aligned(x, xf32 ? 16 : 8)) return fail(MADI_EINVAL, "%s: x must be %d-byte aligned", who, xf32 ? 16 : 8);
    const int ks = gemv_pick_ks(N, K, S.num_sms);
    const bool tile_path =
        aligned(w->qs, 16) && aligned(w->scales, 16) && gemv_tile_ok(m, N, K, xf32 && !x_r16, S.num_sms);
    if (!tile_path && gemv_smem_bytes(m, K, ks, xf32) > (size_t)S.max_smem_optin)
        return fail(MADI_EINVAL, "%s: K=%d too large for the decode path at m=%d", who, K, m);
    GemvArgs a{};
    a.qs = w->qs;
    a.scales = reinterpret_cast<const __half *>(w->scales);
    a.x = x; a.y = y; a.residual = residual; a.bias = bias;
    a.bias_f16 = bias_dtype == MADI_F16;
    a.N = N; a.K = K; a.M = m;
    a.ks = ks;
    cudaError_t e = tile_path
                        ? launch_gemv_tile(a, xf32, y_dtype == MADI_F32, epi, false, S.num_sms, S.dev_err, st, S.pdl,
                                           x_r16)
                        : launch_gemv(a, xf32, y_dtype == MADI_F32, epi, false, st, S.pdl);
    if (e == cudaErrorNotSupported) return fail(MADI_EUNSUPPORTED, "%s: cuTensorMapEncodeTiled unavailable", who);
    if (e != cudaSuccess) return cuda_fail(e, who);
    return MADI_OK;
}

// x_dtype: MADI_F32, MADI_F32_AS_F16 (f32 rounded to f16 as it is loaded) or MADI_F16.
int q8_qkv_impl(const madi_q8w *w, const void *x, int m, const float *qb, const float *vb, float *q_out, float *kc,
                float *vc, const uint32_t *pos, long long cache_stride, cudaStream_t st, const char *who,
                int x_dtype = MADI_F32) {
    const bool x_r16 = x_dtype == MADI_F32_AS_F16, x_f32 = x_dtype != MADI_F16;
    if (!S.ready) return fail(MADI_ENOINIT, "%s: madi_init has not succeeded", who);
    if (!w || !w->qs || !w->scales || !x || !qb || !vb || !q_out || !kc || !vc || !pos)
        return fail(MADI_EINVAL, "%s: null argument", who);
    const int D = w->k;
    if (D <= 0 || D % 32 != 0 || w->n != 3 * D) return fail(MADI_EINVAL, "%s: qkv weight must be [3D][D], D %% 32 == 0", who);
    if (m <= 0 || m > kGemvMaxM) return fail(MADI_EINVAL, "%s: m=%d outside 1..%d", who, m, kGemvMaxM);
    if (!aligned(x, 16) || !aligned(w->qs, 16)) return fail(MADI_EINVAL, "%s: misaligned x or qs", who);
    const int ks = gemv_pick_ks(3 * D, D, S.num_sms);
    const bool tile_path = aligned(w->scales, 16) && gemv_tile_ok(m, 3 * D, D, x_f32 && !x_r16, S.num_sms);
    if (!tile_path && (m > 8 || !x_f32 || x_r16 || gemv_smem_bytes(m, D, ks, true) > (size_t)S.max_smem_optin))
        return fail(MADI_EINVAL, "%s: D=%d at m=%d does not fit the decode path", who, D, m);
    GemvArgs a{};
    a.qs = w->qs;
    a.scales = reinterpret_cast<const __half *>(w->scales);
    a.x = x; a.y = q_out;
    a.N = 3 * D; a.K = D; a.M = m;
    a.ks = ks;
    a.qb = qb; a.vb = vb; a.kc = kc; a.vc = vc; a.pos = pos;
    a.cache_stride = m > 1 ? cache_stride : 0;
    a.D = D;
    cudaError_t e = tile_path ? launch_gemv_tile(a, x_f32, true, MADI_EPI_NONE, true, S.num_sms, S.dev_err, st, S.pdl,
                                                 x_r16)
                              : launch_gemv(a, true, true, MADI_EPI_NONE, true, st, S.pdl);
    if (e == cudaErrorNotSupported) return fail(MADI_EUNSUPPORTED, "%s: cuTensorMapEncodeTiled unavailable", who);
    if (e != cudaSuccess) return cuda_fail(e, who);
    return MADI_OK;
}

// ---------------------------------------------------------------- name table

enum ArgKind { kPtr, kU32, kF32 };
struct ArgVal {
    const void *p;
    uint32_t u;
    float f;
};
using Handler = int (*)(const ArgVal *a, uint32_t gx, cudaStream_t st);   // gx: dispatch grid x

struct Op {
    const char *name;
    std::vector<ArgKind> kinds;
    Handler fn;
};

madi_q8w mkw(const ArgVal &qs, const ArgVal &sc, uint32_t n, uint32_t k) {
    return madi_q8w{static_cast<const int8_t *>(qs.p), static_cast<const uint16_t *>(sc.p), (int32_t)n, (int32_t)k};
}

// gemv_q8(out, qs, scales, x, N, K)  graph_helpers.metal:390-422
int h_gemv(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    madi_q8w w = mkw(a[1], a[2], a[4].u, a[5].u);
    return q8_linear_impl(&w, a[3].p, MADI_F32, 1, nullptr, MADI_F32, MADI_EPI_NONE, nullptr, const_cast<void *>(a[0].p),
                          MADI_F32, st, "gemv_q8");
}
// gemv_q8_bias / _bias_gelu / _bias_res(out, qs, scales, x, bias, N, K)  graph_helpers.metal:424-519
template <int EPI>
int h_gemv_bias(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    madi_q8w w = mkw(a[1], a[2], a[5].u, a[6].u);
    return q8_linear_impl(&w, a[3].p, MADI_F32, 1, a[4].p, MADI_F32, EPI, EPI == MADI_EPI_BIAS_RES ? a[0].p : nullptr,
                          const_cast<void *>(a[0].p), MADI_F32, st, "gemv_q8_bias*");
}
// gemv_q8_qkv(q_out, qs, scales, x, qb, vb, kc, vc, pos_ptr, D)  graph_helpers.metal:527-567
int h_qkv(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    madi_q8w w = mkw(a[1], a[2], 3 * a[9].u, a[9].u);
    return q8_qkv_impl(&w, static_cast<const float *>(a[3].p), 1, static_cast<const float *>(a[4].p),
                       static_cast<const float *>(a[5].p), (float *)a[0].p, (float *)a[6].p, (float *)a[7].p,
                       static_cast<const uint32_t *>(a[8].p), 0, st, "gemv_q8_qkv");
}
// logit_gemv_q8(logits, qs, scales, x, vocab, dim)  graph_helpers.metal:320-352
int h_logit(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    madi_q8w w = mkw(a[1], a[2], a[4].u, a[5].u);
    return q8_linear_impl(&w, a[3].p, MADI_F32, 1, nullptr, MADI_F32, MADI_EPI_NONE, nullptr, const_cast<void *>(a[0].p),
                          MADI_F32, st, "logit_gemv_q8");
}
// dequant_q8_f16(out, qs, scales, N, K)  q8_gemm.metal:12-27
int h_dequant(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    madi_q8w w = mkw(a[1], a[2], a[3].u, a[4].u);
    return madi_q8_dequant_f16(&w, (uint16_t *)a[0].p, st);
}
// mul_mm_q8(C, A, qs, scales, M, N, K)  q8_gemm.metal:29-102
int h_mul_mm(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    madi_q8w w = mkw(a[2], a[3], a[5].u, a[6].u);
    return q8_linear_impl(&w, a[1].p, MADI_F16, (int)a[4].u, nullptr, MADI_F32, MADI_EPI_NONE, nullptr,
                          const_cast<void *>(a[0].p), MADI_F16, st, "mul_mm_q8");
}
// m4_gemm_q8tg / m4_gemm_q8_bias_gelu(A, Wq, scales, C, bias, M, N, K, act_gelu)  m4_gemm.metal:131-266
int h_m4_q8(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    madi_q8w w = mkw(a[1], a[2], a[6].u, a[7].u);
    return q8_linear_impl(&w, a[0].p, MADI_F16, (int)a[5].u, a[4].p, MADI_F32,
                          a[8].u ? MADI_EPI_BIAS_GELU : MADI_EPI_BIAS, nullptr, const_cast<void *>(a[3].p), MADI_F16, st,
                          "m4_gemm_q8");
}

// ---- decode-step primitives by name (graph_helpers.metal); VOCAB = 51866 as in the reference

// Rows of a Q8 table [rows][dim] (+ scales [rows][dim/32]) that both allocations hold.
size_t q8_rows_in(const void *qs, const void *scales, int dim) {
    return std::min(bytes_after(qs) / (size_t)dim, bytes_after(scales) / ((size_t)(dim / 32) * 2));
}
int h_emb_q8_indirect(const ArgVal *a, uint32_t, cudaStream_t st) {      // (out, qs, scales, tokens, pos_ptr, dim)
    const int dim = (int)a[5].u;
    if (dim <= 0 || dim % 32) return fail(MADI_EINVAL, "emb_lookup_indirect_q8: dim %d (multiple of 32)", dim);
    const size_t rows = q8_rows_in(a[1].p, a[2].p, dim), tok_len = bytes_after(a[3].p) / 4;
    if (!rows || !tok_len || bytes_after(a[0].p) < (size_t)dim * 4)
        return fail(MADI_EINVAL, "emb_lookup_indirect_q8: buffer extents unknown or too small");
    cudaError_t e = launch_emb_q8((float *)a[0].p, static_cast<const int8_t *>(a[1].p),
                                  static_cast<const __half *>(a[2].p), static_cast<const uint32_t *>(a[3].p),
                                  static_cast<const uint32_t *>(a[4].p), dim, (int)std::min<size_t>(rows, 1u << 30), 1,
                                  0, (long long)tok_len, nullptr, 0, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "emb_lookup_indirect_q8");
}
int h_emb_q8_direct(const ArgVal *a, uint32_t, cudaStream_t st) {        // (out, qs, scales, tok_ptr, dim)
    const int dim = (int)a[4].u;
    if (dim <= 0 || dim % 32) return fail(MADI_EINVAL, "gpu_emb_lookup_q8: dim %d (multiple of 32)", dim);
    const size_t rows = q8_rows_in(a[1].p, a[2].p, dim);
    if (!rows || bytes_after(a[0].p) < (size_t)dim * 4) return fail(MADI_EINVAL, "gpu_emb_lookup_q8: buffer extents");
    cudaError_t e = launch_emb_q8((float *)a[0].p, static_cast<const int8_t *>(a[1].p),
                                  static_cast<const __half *>(a[2].p), static_cast<const uint32_t *>(a[3].p), nullptr,
                                  dim, (int)std::min<size_t>(rows, 1u << 30), 1, 0, 1, nullptr, 0, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "gpu_emb_lookup_q8");
}
int h_emb_f16_indirect(const ArgVal *a, uint32_t, cudaStream_t st) {     // (out, emb, tokens, pos_ptr, dim)
    const int dim = (int)a[4].u;
    if (dim <= 0) return fail(MADI_EINVAL, "emb_lookup_indirect: dim %d", dim);
    const size_t rows = bytes_after(a[1].p) / ((size_t)dim * 2), tok_len = bytes_after(a[2].p) / 4;
    if (!rows || !tok_len || bytes_after(a[0].p) < (size_t)dim * 4)
        return fail(MADI_EINVAL, "emb_lookup_indirect: buffer extents unknown or too small");
    cudaError_t e = launch_emb_f16((float *)a[0].p, static_cast<const __half *>(a[1].p),
                                   static_cast<const uint32_t *>(a[2].p), static_cast<const uint32_t *>(a[3].p), dim,
                                   (int)std::min<size_t>(rows, 1u << 30), (long long)tok_len, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "emb_lookup_indirect");
}
int h_pos_add(const ArgVal *a, uint32_t, cudaStream_t st) {              // (out, pos_emb, pos_ptr, dim)
    const int dim = (int)a[3].u;
    if (dim <= 0) return fail(MADI_EINVAL, "pos_embed_add_indirect: dim %d", dim);
    const size_t max_pos = bytes_after(a[1].p) / ((size_t)dim * 4);
    if (!max_pos || bytes_after(a[0].p) < (size_t)dim * 4) return fail(MADI_EINVAL, "pos_embed_add_indirect: extents");
    cudaError_t e = launch_pos_add((float *)a[0].p, static_cast<const float *>(a[1].p),
                                   static_cast<const uint32_t *>(a[2].p), dim, (int)std::min<size_t>(max_pos, 1u << 30),
                                   st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "pos_embed_add_indirect");
}
int h_step_advance(const ArgVal *a, uint32_t, cudaStream_t st) {         // (pos_ptr)
    cudaError_t e = launch_step_advance((uint32_t *)a[0].p, 1, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "step_advance");
}
template <bool kConf>
int h_argmax(const ArgVal *a, uint32_t, cudaStream_t st) {   // (logits, tokens, [conf,] pos_ptr, max_len)
    const int i_pos = kConf ? 3 : 2;
    const uint32_t max_len = a[i_pos + 1].u;
    if (bytes_after(a[0].p) < (size_t)kWhisperVocab * 4) return fail(MADI_EINVAL, "argmax: logits shorter than VOCAB");
    if (bytes_after(a[1].p) < (size_t)max_len * 4 || (kConf && bytes_after(a[2].p) < (size_t)max_len * 4))
        return fail(MADI_EINVAL, "argmax: tokens / conf shorter than max_len");
    cudaError_t e = launch_argmax(static_cast<const float *>(a[0].p), (uint32_t *)a[1].p, kConf ? (float *)a[2].p : nullptr,
                                  static_cast<const uint32_t *>(a[i_pos].p), kWhisperVocab, (int)max_len, 1, 0, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "argmax");
}
int h_suppress(const ArgVal *a, uint32_t, cudaStream_t st) {             // (logits, ids, n)
    const uint32_t n = a[2].u;
    if (bytes_after(a[0].p) < (size_t)kWhisperVocab * 4 || bytes_after(a[1].p) < (size_t)n * 4)
        return fail(MADI_EINVAL, "suppress_list: buffer extents");
    cudaError_t e =
        launch_suppress((float *)a[0].p, static_cast<const uint32_t *>(a[1].p), (int)n, kWhisperVocab, 1, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "suppress_list");
}
// (logits, past_tokens, num_suppress, step_ptr, sample_begin, no_repeat_ngram)
int h_logit_filter(const ArgVal *a, uint32_t, cudaStream_t st) {
    if (bytes_after(a[0].p) < (size_t)kWhisperVocab * 4) return fail(MADI_EINVAL, "logit_filter_indirect: logits");
    const size_t past_len = bytes_after(a[1].p) / 4;
    cudaError_t e = launch_logit_filter((float *)a[0].p, static_cast<const uint32_t *>(a[1].p),
                                        static_cast<const uint32_t *>(a[3].p), a[4].u, a[5].u, kWhisperVocab,
                                        (int)std::min<size_t>(past_len, 1u << 30), 1, 0, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "logit_filter_indirect");
}

// m4_flash_enc(out, q, k, v, seq_len, nh): packed [seq][nh*64] f16 buffers   m4_gemm.metal:268-407
int h_flash_enc(const ArgVal *a, uint32_t, cudaStream_t st) {
    const uint32_t seq = a[4].u, nh = a[5].u;
    if (seq == 0 || seq > (1u << 20) || nh == 0 || nh > 1024) return fail(MADI_EINVAL, "m4_flash_enc: seq %u, heads %u", seq, nh);
    const size_t bytes = (size_t)seq * nh * 64 * 2;
    for (int i = 0; i < 4; ++i)
        if (!a[i].p || !aligned(a[i].p, 16) || bytes_after(a[i].p) < bytes)
            return fail(MADI_EINVAL, "m4_flash_enc: buffer %d extent / alignment", i);
    return madi_flash_attn_enc(static_cast<const uint16_t *>(a[1].p), static_cast<const uint16_t *>(a[2].p),
                               static_cast<const uint16_t *>(a[3].p), (int)nh * 64, (uint16_t *)a[0].p, (int)nh * 64,
                               (int)seq, (int)nh, 1, st);
}

// bias_res_ln(X, MO, bias, Y, gamma, beta, D, eps) / layer_norm(X, Y, gamma, beta, D, eps), f32, rows = grid x
//   encoder_ops.metal:14-120 (the decoder's LayerNorms)
int h_bias_res_ln_f32(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    return madi_bias_res_ln((float *)a[0].p, static_cast<const float *>(a[1].p), static_cast<const float *>(a[2].p),
                            (float *)a[3].p, static_cast<const float *>(a[4].p), static_cast<const float *>(a[5].p),
                            (int)gx, (int)a[6].u, a[7].f, st);
}
int h_layer_norm_f32(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    return madi_layer_norm(static_cast<const float *>(a[0].p), (float *)a[1].p, static_cast<const float *>(a[2].p),
                           static_cast<const float *>(a[3].p), (int)gx, (int)a[4].u, a[5].f, st);
}

// ---- decoder attention by name (decoder_ops.metal:81-531); head_dim 64, K/V rows
// of kvd elements, head h reading the kv head h * nkv / nh.  Buffer extents come
// from the allocations (the reference signatures carry none) and bound every read.
int attn_shape_ok(const char *who, uint32_t hdd, uint32_t kvd, uint32_t nkv, uint32_t nh) {
    if (hdd != 64) return fail(MADI_EINVAL, "%s: head_dim %u (64 supported)", who, hdd);
    if (nh == 0 || nh > 1024 || nkv == 0 || nkv > nh || (size_t)kvd < (size_t)nkv * 64 || kvd % 8)
        return fail(MADI_EINVAL, "%s: heads %u, kv heads %u, kv_dim %u", who, nh, nkv, kvd);
    return MADI_OK;
}
bool extent_ok(const void *p, size_t bytes) { return p && aligned(p, 16) && bytes_after(p) >= bytes; }

// gpu_attention(out, q, kc, vc, pos_ptr, hdd, kvd, nkv, nh): f32 cache, one slot
int h_self_attn(const ArgVal *a, uint32_t, cudaStream_t st) {
    const uint32_t hdd = a[5].u, kvd = a[6].u, nkv = a[7].u, nh = a[8].u;
    if (int rc = attn_shape_ok("gpu_attention", hdd, kvd, nkv, nh)) return rc;
    const size_t row = (size_t)kvd * 4, qb = (size_t)nh * 64 * 4;
    const size_t rows = std::min(bytes_after(a[2].p), bytes_after(a[3].p)) / row;
    if (!rows || !extent_ok(a[0].p, qb) || !extent_ok(a[1].p, qb) || !aligned(a[2].p, 16) || !aligned(a[3].p, 16))
        return fail(MADI_EINVAL, "gpu_attention: buffer extents");
    const int max_tok = (int)std::min<size_t>(rows, kAttnMaxTok);
    cudaError_t e = launch_self_attn((float *)a[0].p, static_cast<const float *>(a[1].p), a[2].p, a[3].p, false,
                                     static_cast<const uint32_t *>(a[4].p), 1, (int)kvd, (int)nkv, (int)nh, max_tok,
                                     S.dev_err, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "gpu_attention");
}
// flash_cross_attn (f32 K/V) / flash_cross_attn_f16kv (+ sc_out, write_sc) /
// flash_cross_attn_f16kv_batched (slots = grid x / nh)
template <bool kF16, int kMode>   // kMode 0: one slot; 1: with scores; 2: batched
int h_cross_attn(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    const char *who = kMode == 2 ? "flash_cross_attn_f16kv_batched" : kF16 ? "flash_cross_attn_f16kv" : "flash_cross_attn";
    const uint32_t seqlen = a[4].u, hdd = a[5].u, kvd = a[6].u, nkv = a[7].u, nh = a[8].u;
    if (int rc = attn_shape_ok(who, hdd, kvd, nkv, nh)) return rc;
    if (seqlen == 0 || attn_cluster_size((int)seqlen) == 0) return fail(MADI_EINVAL, "%s: seqlen %u", who, seqlen);
    const uint32_t slots = kMode == 2 ? gx / nh : 1;
    if (slots == 0 || (kMode == 2 && gx % nh)) return fail(MADI_EINVAL, "%s: grid x %u is not slots x %u heads", who, gx, nh);
    const size_t kvb = (size_t)slots * seqlen * kvd * (kF16 ? 2 : 4), qb = (size_t)slots * nh * 64 * 4;
    if (!extent_ok(a[0].p, qb) || !extent_ok(a[1].p, qb) || !extent_ok(a[2].p, kvb) || !extent_ok(a[3].p, kvb))
        return fail(MADI_EINVAL, "%s: buffer extents", who);
    float *scores = nullptr;
    if (kMode == 1 && a[10].u) {
        if (!extent_ok(a[9].p, (size_t)nh * seqlen * 4)) return fail(MADI_EINVAL, "%s: sc_out extent", who);
        scores = (float *)a[9].p;
    }
    cudaError_t e = launch_cross_attn((float *)a[0].p, static_cast<const float *>(a[1].p), a[2].p, a[3].p, kF16, scores,
                                      (int)slots, (int)seqlen, (int)kvd, (int)nkv, (int)nh, S.dev_err, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, who);
}
// flash_cross_attn_split(part, q, kc, vc, seqlen, hdd, kvd, nkv, nh, nsplit, sc_raw, write_sc), grid nh * nsplit
int h_cross_split(const ArgVal *a, uint32_t, cudaStream_t st) {
    const uint32_t seqlen = a[4].u, hdd = a[5].u, kvd = a[6].u, nkv = a[7].u, nh = a[8].u, nsplit = a[9].u;
    if (int rc = attn_shape_ok("flash_cross_attn_split", hdd, kvd, nkv, nh)) return rc;
    if (seqlen == 0 || nsplit == 0 || nsplit > 1024 || (seqlen + nsplit - 1) / nsplit > (uint32_t)kAttnMaxChunk)
        return fail(MADI_EINVAL, "flash_cross_attn_split: seqlen %u over %u splits", seqlen, nsplit);
    const size_t kvb = (size_t)seqlen * kvd * 2;
    if (!extent_ok(a[0].p, (size_t)nh * nsplit * 66 * 4) || !extent_ok(a[1].p, (size_t)nh * 256) ||
        !extent_ok(a[2].p, kvb) || !extent_ok(a[3].p, kvb) || (a[11].u && !extent_ok(a[10].p, (size_t)nh * seqlen * 4)))
        return fail(MADI_EINVAL, "flash_cross_attn_split: buffer extents");
    cudaError_t e = launch_cross_attn_part((float *)a[0].p, static_cast<const float *>(a[1].p), a[2].p, a[3].p, true,
                                           (float *)a[10].p, (int)(a[11].u != 0), (int)seqlen, (int)kvd, (int)nkv,
                                           (int)nh, (int)nsplit, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "flash_cross_attn_split");
}
// flash_cross_attn_reduce(out, part, hdd, nsplit, sc_out, seqlen, write_sc), heads = grid x
int h_cross_reduce(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    const uint32_t hdd = a[2].u, nsplit = a[3].u, seqlen = a[5].u, nh = gx;
    if (hdd != 64 || nh == 0 || nh > 1024 || nsplit == 0 || nsplit > 1024)
        return fail(MADI_EINVAL, "flash_cross_attn_reduce: head_dim %u, heads %u, splits %u", hdd, nh, nsplit);
    if (!extent_ok(a[0].p, (size_t)nh * 256) || !extent_ok(a[1].p, (size_t)nh * nsplit * 66 * 4) ||
        (a[6].u && !extent_ok(a[4].p, (size_t)nh * seqlen * 4)))
        return fail(MADI_EINVAL, "flash_cross_attn_reduce: buffer extents");
    cudaError_t e = launch_cross_attn_reduce((float *)a[0].p, static_cast<const float *>(a[1].p), (int)nsplit,
                                             (float *)a[4].p, (int)seqlen, (int)(a[6].u != 0), (int)nh, st);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "flash_cross_attn_reduce");
}

// bias_res_ln_f16(X, MO, bias, Y, gamma, beta, D, eps), rows = grid x   encoder_ops.metal:333-364
int h_bias_res_ln(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    return madi_bias_res_ln_f16((float *)a[0].p, static_cast<const uint16_t *>(a[1].p), static_cast<const float *>(a[2].p),
                                (uint16_t *)a[3].p, static_cast<const float *>(a[4].p), static_cast<const float *>(a[5].p),
                                (int)gx, (int)a[6].u, a[7].f, st);
}
// layer_norm_f16(X, Y, gamma, beta, D, eps), rows = grid x   encoder_ops.metal:305-331
int h_layer_norm(const ArgVal *a, uint32_t gx, cudaStream_t st) {
    return madi_layer_norm_f16(static_cast<const float *>(a[0].p), (uint16_t *)a[1].p, static_cast<const float *>(a[2].p),
                               static_cast<const float *>(a[3].p), (int)gx, (int)a[4].u, a[5].f, st);
}

const std::vector<Op> &ops() {
    static const std::vector<Op> table = {
        {"gemv_q8", {kPtr, kPtr, kPtr, kPtr, kU32, kU32}, h_gemv},
        {"gemv_q8_bias", {kPtr, kPtr, kPtr, kPtr, kPtr, kU32, kU32}, h_gemv_bias<MADI_EPI_BIAS>},
        {"gemv_q8_bias_gelu", {kPtr, kPtr, kPtr, kPtr, kPtr, kU32, kU32}, h_gemv_bias<MADI_EPI_BIAS_GELU>},
        {"gemv_q8_bias_res", {kPtr, kPtr, kPtr, kPtr, kPtr, kU32, kU32}, h_gemv_bias<MADI_EPI_BIAS_RES>},
        {"gemv_q8_qkv", {kPtr, kPtr, kPtr, kPtr, kPtr, kPtr, kPtr, kPtr, kPtr, kU32}, h_qkv},
        {"logit_gemv_q8", {kPtr, kPtr, kPtr, kPtr, kU32, kU32}, h_logit},
        {"dequant_q8_f16", {kPtr, kPtr, kPtr, kU32, kU32}, h_dequant},
        {"mul_mm_q8", {kPtr, kPtr, kPtr, kPtr, kU32, kU32, kU32}, h_mul_mm},
        {"m4_gemm_q8tg", {kPtr, kPtr, kPtr, kPtr, kPtr, kU32, kU32, kU32, kU32}, h_m4_q8},
        {"m4_gemm_q8_bias_gelu", {kPtr, kPtr, kPtr, kPtr, kPtr, kU32, kU32, kU32, kU32}, h_m4_q8},
        {"bias_res_ln_f16", {kPtr, kPtr, kPtr, kPtr, kPtr, kPtr, kU32, kF32}, h_bias_res_ln},
        {"layer_norm_f16", {kPtr, kPtr, kPtr, kPtr, kU32, kF32}, h_layer_norm},
        {"bias_res_ln", {kPtr, kPtr, kPtr, kPtr, kPtr, kPtr, kU32, kF32}, h_bias_res_ln_f32},
        {"layer_norm", {kPtr, kPtr, kPtr, kPtr, kU32, kF32}, h_layer_norm_f32},
        {"emb_lookup_indirect_q8", {kPtr, kPtr, kPtr, kPtr, kPtr, kU32}, h_emb_q8_indirect},
        {"gpu_emb_lookup_q8", {kPtr, kPtr, kPtr, kPtr, kU32}, h_emb_q8_direct},
        {"emb_lookup_indirect", {kPtr, kPtr, kPtr, kPtr, kU32}, h_emb_f16_indirect},
        {"pos_embed_add_indirect", {kPtr, kPtr, kPtr, kU32}, h_pos_add},
        {"step_advance", {kPtr}, h_step_advance},
        {"argmax_no_inc", {kPtr, kPtr, kPtr, kU32}, h_argmax<false>},
        {"argmax_conf", {kPtr, kPtr, kPtr, kPtr, kU32}, h_argmax<true>},
        {"suppress_list", {kPtr, kPtr, kU32}, h_suppress},
        {"logit_filter_indirect", {kPtr, kPtr, kU32, kPtr, kU32, kU32}, h_logit_filter},
        {"gpu_attention", {kPtr, kPtr, kPtr, kPtr, kPtr, kU32, kU32, kU32, kU32}, h_self_attn},
        {"flash_cross_attn", {kPtr, kPtr, kPtr, kPtr, kU32, kU32, kU32, kU32, kU32}, h_cross_attn<false, 0>},
        {"flash_cross_attn_f16kv", {kPtr, kPtr, kPtr, kPtr, kU32, kU32, kU32, kU32, kU32, kPtr, kU32},
         h_cross_attn<true, 1>},
        {"flash_cross_attn_f16kv_batched", {kPtr, kPtr, kPtr, kPtr, kU32, kU32, kU32, kU32, kU32},
         h_cross_attn<true, 2>},
        {"flash_cross_attn_split", {kPtr, kPtr, kPtr, kPtr, kU32, kU32, kU32, kU32, kU32, kU32, kPtr, kU32},
         h_cross_split},
        {"flash_cross_attn_reduce", {kPtr, kPtr, kU32, kU32, kPtr, kU32, kU32}, h_cross_reduce},
        {"m4_flash_enc", {kPtr, kPtr, kPtr, kPtr, kU32, kU32}, h_flash_enc},
    };
    return table;
}

void prof_add(const char *name, double ms) {
    auto &e = S.prof[name];
    e.first += 1;
    e.second += ms;
}

}  // namespace

// ======================================================================= C ABI
extern "C" {

int madi_init(int device) {
    if (S.ready) {
        if (device == S.device) return MADI_OK;
        return fail(MADI_EBUSY, "madi_init: already bound to device %d", S.device);
    }
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) { cudaGetLastError(); return cuda_fail(e, "madi_init: cudaGetDeviceCount"); }
    if (device < 0 || device >= n) return fail(MADI_EINVAL, "madi_init: device %d of %d", device, n);
    if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "madi_init: cudaSetDevice");
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return cuda_fail(e, "madi_init: properties");
    if (prop.major != 10 || prop.minor != 0)
        return fail(MADI_EUNSUPPORTED, "madi_init: %s is sm_%d%d; this library is built for sm_100a", prop.name,
                    prop.major, prop.minor);
    S.device = device;
    S.num_sms = prop.multiProcessorCount;
    cudaDeviceGetAttribute(&S.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    // a BLOCKING stream: it orders against the legacy default stream, so work
    // a caller (e.g. torch) queued there is visible to our kernels and vice versa
    if ((e = cudaStreamCreateWithFlags(&S.own_stream, cudaStreamDefault)) != cudaSuccess)
        return cuda_fail(e, "madi_init: stream");
    S.stream = S.own_stream;
    if ((e = cudaMalloc(&S.dev_err, 256)) != cudaSuccess) return cuda_fail(e, "madi_init: error word");
    cudaMemset(S.dev_err, 0, 256);
    if ((e = cudaEventCreateWithFlags(&S.done, cudaEventDisableTiming)) != cudaSuccess)
        return cuda_fail(e, "madi_init: event");
    const char *pv = getenv("MADI_PROFILE");
    S.profile = pv && pv[0] == '1';
    const char *pd = getenv("MADI_PDL");
    S.pdl = !(pd && pd[0] == '0');
    const char *dv = getenv("MADI_DEBUG");
    if (dv && dv[0] == '1') S.verbose = 1;
    if (!tensor_map_encoder()) return fail(MADI_EUNSUPPORTED, "madi_init: cuTensorMapEncodeTiled unavailable");
    cudaDeviceSynchronize();
    S.ready = true;
    if (S.verbose) fprintf(stderr, "[madi] device %d %s, %d SMs\n", device, prop.name, S.num_sms);
    return MADI_OK;
}

void madi_cleanup(void) {
    if (!S.ready) return;
    if (S.capturing) {
        cudaGraph_t g = nullptr;
        cudaStreamEndCapture(S.stream, &g);
        if (g) cudaGraphDestroy(g);
        S.capturing = false;
    }
    cudaStreamSynchronize(S.stream);
    if (S.exec) cudaGraphExecDestroy(S.exec);
    if (S.done) cudaEventDestroy(S.done);
    if (S.dev_err) cudaFree(S.dev_err);
    if (S.own_stream) cudaStreamDestroy(S.own_stream);
    {
        std::lock_guard<std::mutex> lk(g_alloc_mu);
        for (auto &kv : g_allocs) cudaFree(reinterpret_cast<void *>(kv.first));
        g_allocs.clear();
    }
    forget_split_static_addresses();
    S = State();
}

void *madi_alloc(size_t size) {
    if (!S.ready) { fail(MADI_ENOINIT, "madi_alloc: not initialised"); return nullptr; }
    if (size == 0) size = 1;
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size + 255) & ~size_t(255));
    if (e != cudaSuccess) { cuda_fail(e, "madi_alloc"); return nullptr; }
    std::lock_guard<std::mutex> lk(g_alloc_mu);
    g_allocs[reinterpret_cast<uintptr_t>(p)] = size;
    return p;
}

void madi_free(void *ptr) {
    if (!ptr) return;
    {
        std::lock_guard<std::mutex> lk(g_alloc_mu);
        auto it = g_allocs.find(reinterpret_cast<uintptr_t>(ptr));
        if (it == g_allocs.end()) { fail(MADI_EINVAL, "madi_free: %p was not returned by madi_alloc", ptr); return; }
        g_allocs.erase(it);
    }
    cudaFree(ptr);
}

int madi_upload(void *dst, const void *src, size_t size) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_upload: not initialised");
    if (!dst || !src) return fail(MADI_EINVAL, "madi_upload: null pointer");
    cudaError_t e = cudaMemcpyAsync(dst, src, size, cudaMemcpyHostToDevice, S.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(S.stream);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_upload");
}

int madi_download(void *dst, const void *src, size_t size) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_download: not initialised");
    if (!dst || !src) return fail(MADI_EINVAL, "madi_download: null pointer");
    cudaError_t e = cudaMemcpyAsync(dst, src, size, cudaMemcpyDeviceToHost, S.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(S.stream);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_download");
}

int madi_get_function(const char *name, int *out_id) {
    if (!name || !out_id) return fail(MADI_EINVAL, "madi_get_function: null argument");
    const auto &t = ops();
    for (size_t i = 0; i < t.size(); ++i)
        if (strcmp(t[i].name, name) == 0) { *out_id = (int)i; return MADI_OK; }
    return fail(MADI_ENOTFOUND, "madi_get_function: no kernel named '%s'", name);
}

int madi_dispatch(int func_id, uint32_t gx, uint32_t gy, uint32_t gz, uint32_t bx, uint32_t by, uint32_t bz,
                  const void **args, const size_t *arg_sizes, int n_args) {
    (void)gy; (void)gz; (void)bx; (void)by; (void)bz;   // gx: row count of the LayerNorm kernels
    if (!S.ready) return fail(MADI_ENOINIT, "madi_dispatch: not initialised");
    const auto &t = ops();
    if (func_id < 0 || func_id >= (int)t.size()) return fail(MADI_EINVAL, "madi_dispatch: bad function id %d", func_id);
    const Op &op = t[func_id];
    if (n_args != (int)op.kinds.size())
        return fail(MADI_EINVAL, "madi_dispatch(%s): %d arguments, expected %zu", op.name, n_args, op.kinds.size());
    if (!args || !arg_sizes) return fail(MADI_EINVAL, "madi_dispatch(%s): null argument arrays", op.name);
    ArgVal v[16];
    for (int i = 0; i < n_args; ++i) {
        if (!args[i]) return fail(MADI_EINVAL, "madi_dispatch(%s): argument %d is null", op.name, i);
        switch (op.kinds[i]) {
            case kPtr:
                if (arg_sizes[i] != sizeof(void *))
                    return fail(MADI_EINVAL, "madi_dispatch(%s): argument %d must be a buffer pointer", op.name, i);
                memcpy(&v[i].p, args[i], sizeof(void *));
                if (!is_device_ptr(v[i].p))
                    return fail(MADI_EINVAL, "madi_dispatch(%s): argument %d (%p) is not device memory", op.name, i,
                                v[i].p);
                break;
            case kU32:
                if (arg_sizes[i] != 4) return fail(MADI_EINVAL, "madi_dispatch(%s): argument %d must be u32", op.name, i);
                memcpy(&v[i].u, args[i], 4);
                break;
            case kF32:
                if (arg_sizes[i] != 4) return fail(MADI_EINVAL, "madi_dispatch(%s): argument %d must be f32", op.name, i);
                memcpy(&v[i].f, args[i], 4);
                break;
        }
    }
    if (S.profile && !S.capturing) {
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, S.stream);
        int rc = op.fn(v, gx, S.stream);
        cudaEventRecord(e1, S.stream);
        cudaEventSynchronize(e1);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        if (rc == MADI_OK) prof_add(op.name, ms);
        return rc;
    }
    return op.fn(v, gx, S.stream);
}

int madi_begin_command_buffer(void) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_begin_command_buffer: not initialised");
    if (S.capturing) return fail(MADI_EBUSY, "madi_begin_command_buffer: a command buffer is already open");
    cudaError_t e = cudaStreamBeginCapture(S.stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return cuda_fail(e, "madi_begin_command_buffer");
    S.capturing = true;
    return MADI_OK;
}

int madi_commit_command_buffer(void) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_commit_command_buffer: not initialised");
    if (!S.capturing) return fail(MADI_EBUSY, "madi_commit_command_buffer: no command buffer open");
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(S.stream, &g);
    S.capturing = false;
    if (e != cudaSuccess) return cuda_fail(e, "madi_commit_command_buffer: end capture");
    if (S.exec) {
        cudaGraphExecUpdateResultInfo info;
        if (cudaGraphExecUpdate(S.exec, g, &info) != cudaSuccess) {
            cudaGetLastError();
            cudaGraphExecDestroy(S.exec);
            S.exec = nullptr;
        }
    }
    if (!S.exec && (e = cudaGraphInstantiate(&S.exec, g, 0)) != cudaSuccess) {
        cudaGraphDestroy(g);
        return cuda_fail(e, "madi_commit_command_buffer: instantiate");
    }
    cudaGraphDestroy(g);
    if ((e = cudaGraphLaunch(S.exec, S.stream)) != cudaSuccess) return cuda_fail(e, "madi_commit_command_buffer: launch");
    return MADI_OK;
}

void madi_flush(void) {}

int madi_sync(int timeout_ms) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_sync: not initialised");
    if (S.capturing) return fail(MADI_EBUSY, "madi_sync: a command buffer is open (commit it first)");
    cudaError_t e = cudaEventRecord(S.done, S.stream);
    if (e != cudaSuccess) return cuda_fail(e, "madi_sync: record");
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        e = cudaEventQuery(S.done);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_fail(e, "madi_sync");
        if (timeout_ms >= 0 &&
            std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
            return fail(MADI_ETIMEDOUT, "madi_sync: work still pending after %d ms", timeout_ms);
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    int word = 0;
    if ((e = cudaMemcpy(&word, S.dev_err, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "madi_sync: error word");
    if (word != 0) {
        cudaMemset(S.dev_err, 0, sizeof(int));
        return fail(MADI_EDEVICE, "madi_sync: a kernel reported device error %d (bounded wait expired)", word);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "madi_sync");
    return MADI_OK;
}

int madi_set_stream(void *cuda_stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_set_stream: not initialised");
    if (S.capturing) return fail(MADI_EBUSY, "madi_set_stream: a command buffer is open");
    S.stream = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : S.own_stream;
    return MADI_OK;
}

void *madi_get_stream(void) { return S.stream; }

const char *madi_last_error(void) { return g_last_error.c_str(); }

void madi_set_verbose(int v) { S.verbose = v; }

int madi_num_sms(void) { return S.num_sms; }

void madi_dump_profile(const char *out_path) {
    FILE *f = out_path ? fopen(out_path, "w") : stdout;
    if (!f) return;
    double total = 0;
    std::vector<std::pair<std::string, std::pair<long long, double>>> rows(S.prof.begin(), S.prof.end());
    for (auto &r : rows) total += r.second.second;
    std::sort(rows.begin(), rows.end(), [](auto &a, auto &b) { return a.second.second > b.second.second; });
    fprintf(f, " Time (%%)  Total Time (ns)  Instances  Avg (ns)  Name\n");
    for (auto &r : rows) {
        const double ns = r.second.second * 1e6;
        fprintf(f, " %7.1f  %15.0f  %9lld  %8.0f  %s\n", total > 0 ? 100.0 * r.second.second / total : 0.0, ns,
                r.second.first, ns / (double)r.second.first, r.first.c_str());
    }
    if (f != stdout) fclose(f);
}

int madi_q8_linear(const madi_q8w *w, const void *x, int x_dtype, int m, const void *bias, int bias_dtype, int epi,
                   const void *residual, void *y, int y_dtype, void *stream) {
    return q8_linear_impl(w, x, x_dtype, m, bias, bias_dtype, epi, residual, y, y_dtype, pick_stream(stream),
                          "madi_q8_linear");
}

int madi_q8_qkv(const madi_q8w *w, const float *x, int m, const float *qb, const float *vb, float *q_out, float *kc,
                float *vc, const uint32_t *pos, int64_t cache_stride, void *stream) {
    return q8_qkv_impl(w, x, m, qb, vb, q_out, kc, vc, pos, (long long)cache_stride, pick_stream(stream), "madi_q8_qkv",
                       MADI_F32);
}

int madi_q8_qkv_ex(const madi_q8w *w, const void *x, int x_dtype, int m, const float *qb, const float *vb,
                   float *q_out, float *kc, float *vc, const uint32_t *pos, int64_t cache_stride, void *stream) {
    if (x_dtype != MADI_F32 && x_dtype != MADI_F32_AS_F16 && x_dtype != MADI_F16)
        return fail(MADI_EINVAL, "madi_q8_qkv_ex: x_dtype %d (MADI_F32, MADI_F16 or MADI_F32_AS_F16)", x_dtype);
    return q8_qkv_impl(w, x, m, qb, vb, q_out, kc, vc, pos, (long long)cache_stride, pick_stream(stream),
                       "madi_q8_qkv_ex", x_dtype);
}

int madi_q8_dequant_f16(const madi_q8w *w, uint16_t *out, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_q8_dequant_f16: not initialised");
    if (!w || !w->qs || !w->scales || !out) return fail(MADI_EINVAL, "madi_q8_dequant_f16: null argument");
    if (w->n <= 0 || w->k <= 0 || w->k % 32) return fail(MADI_EINVAL, "madi_q8_dequant_f16: bad shape");
    if (!aligned(w->qs, 16) || !aligned(out, 16)) return fail(MADI_EINVAL, "madi_q8_dequant_f16: misaligned buffer");
    cudaError_t e = launch_dequant_f16(w->qs, reinterpret_cast<const __half *>(w->scales), w->n, w->k,
                                       reinterpret_cast<__half *>(out), pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_q8_dequant_f16");
}

int madi_q8_quantize_f16(const uint16_t *w, int rows, int dim, int8_t *qs, uint16_t *scales, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_q8_quantize_f16: not initialised");
    if (!w || !qs || !scales) return fail(MADI_EINVAL, "madi_q8_quantize_f16: null argument");
    if (rows <= 0 || dim <= 0 || dim % 32) return fail(MADI_EINVAL, "madi_q8_quantize_f16: bad shape (dim %% 32)");
    cudaError_t e = launch_quantize_f16(reinterpret_cast<const __half *>(w), rows, dim, qs,
                                        reinterpret_cast<__half *>(scales), pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_q8_quantize_f16");
}

namespace {
// Operand types: kLnF16 MO and Y f16 (the encoder's *_f16 forms); kLnF32 MO and Y f32
// (the decoder's); kLnF32Y16 MO f32, Y f16 (the decoder's, feeding f16 activations).
enum LnTypes { kLnF16 = 0, kLnF32 = 1, kLnF32Y16 = 2 };
int res_ln_impl(float *x, const void *mo, const float *bias, void *y, const float *gamma, const float *beta, int rows,
                int d, float eps, void *stream, const char *who, int types = kLnF16) {
    if (!S.ready) return fail(MADI_ENOINIT, "%s: not initialised", who);
    if (!x || !y || !gamma || !beta || (mo && !bias)) return fail(MADI_EINVAL, "%s: null argument", who);
    if (rows < 0 || d < 128 || d > kLnMaxD || d % 128)
        return fail(MADI_EINVAL, "%s: rows=%d, D=%d (need 128 <= D <= %d, D %% 128 == 0)", who, rows, d, kLnMaxD);
    if (!(eps >= 0.f) || eps > 1.f) return fail(MADI_EINVAL, "%s: eps=%g", who, (double)eps);
    const size_t ya = types == kLnF32 ? 16 : 8, ma = types == kLnF16 ? 8 : 16;
    if (!aligned(x, 16) || !aligned(gamma, 16) || !aligned(beta, 16) || !aligned(y, ya) || (mo && !aligned(mo, ma)) ||
        (bias && !aligned(bias, 16)))
        return fail(MADI_EINVAL, "%s: misaligned buffer (f32 rows 16-byte, f16 rows 8-byte aligned)", who);
    if ((size_t)rows * (size_t)d >= (1ull << 31)) return fail(MADI_EINVAL, "%s: too large", who);
    if (rows == 0) return MADI_OK;
    cudaError_t e =
        types == kLnF32    ? launch_res_ln_f32(x, static_cast<const float *>(mo), bias, static_cast<float *>(y), gamma,
                                               beta, rows, d, eps, pick_stream(stream))
        : types == kLnF32Y16 ? launch_res_ln_f32_y16(x, static_cast<const float *>(mo), bias, static_cast<__half *>(y),
                                                   gamma, beta, rows, d, eps, pick_stream(stream))
                           : launch_res_ln(x, static_cast<const __half *>(mo), bias, static_cast<__half *>(y), gamma,
                                           beta, rows, d, eps, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, who);
}
}  // namespace

int madi_bias_res_ln(float *x, const float *mo, const float *bias, float *y, const float *gamma, const float *beta,
                     int rows, int d, float eps, void *stream) {
    if (!mo) return fail(MADI_EINVAL, "madi_bias_res_ln: null MO");
    return res_ln_impl(x, mo, bias, y, gamma, beta, rows, d, eps, stream, "madi_bias_res_ln", kLnF32);
}

int madi_layer_norm(const float *x, float *y, const float *gamma, const float *beta, int rows, int d, float eps,
                    void *stream) {
    return res_ln_impl(const_cast<float *>(x), nullptr, nullptr, y, gamma, beta, rows, d, eps, stream, "madi_layer_norm",
                       kLnF32);
}

int madi_bias_res_ln_y16(float *x, const float *mo, const float *bias, uint16_t *y, const float *gamma,
                         const float *beta, int rows, int d, float eps, void *stream) {
    if (!mo) return fail(MADI_EINVAL, "madi_bias_res_ln_y16: null MO");
    return res_ln_impl(x, mo, bias, y, gamma, beta, rows, d, eps, stream, "madi_bias_res_ln_y16", kLnF32Y16);
}

int madi_layer_norm_y16(const float *x, uint16_t *y, const float *gamma, const float *beta, int rows, int d, float eps,
                        void *stream) {
    return res_ln_impl(const_cast<float *>(x), nullptr, nullptr, y, gamma, beta, rows, d, eps, stream,
                       "madi_layer_norm_y16", kLnF32Y16);
}

int madi_bias_res_ln_f16(float *x, const uint16_t *mo, const float *bias, uint16_t *y, const float *gamma,
                         const float *beta, int rows, int d, float eps, void *stream) {
    if (!mo) return fail(MADI_EINVAL, "madi_bias_res_ln_f16: null MO");
    return res_ln_impl(x, mo, bias, y, gamma, beta, rows, d, eps, stream, "madi_bias_res_ln_f16");
}

static int emb_impl(const madi_q8w *emb, const uint32_t *tokens, const uint32_t *pos, int m, int64_t tok_stride,
                    int tok_len, const float *pos_emb, int max_pos, float *out, void *stream, const char *what) {
    if (!S.ready) return fail(MADI_ENOINIT, "%s: not initialised", what);
    if (!emb || !emb->qs || !emb->scales || !tokens || !out) return fail(MADI_EINVAL, "%s: null argument", what);
    if (emb->n <= 0 || emb->k <= 0 || emb->k % 32 || m <= 0 || m > 65535 || tok_len <= 0 ||
        (m > 1 && pos && tok_stride < tok_len))
        return fail(MADI_EINVAL, "%s: bad shape (rows=%d dim=%d m=%d tok_len=%d)", what, emb->n, emb->k, m, tok_len);
    cudaError_t e = launch_emb_q8(out, emb->qs, reinterpret_cast<const __half *>(emb->scales), tokens, pos, emb->k,
                                  emb->n, m, pos ? (long long)tok_stride : 1, pos ? (long long)tok_len : 1, pos_emb,
                                  max_pos, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, what);
}

int madi_emb_lookup_q8(const madi_q8w *emb, const uint32_t *tokens, const uint32_t *pos, int m, int64_t tok_stride,
                       int tok_len, float *out, void *stream) {
    return emb_impl(emb, tokens, pos, m, tok_stride, tok_len, nullptr, 0, out, stream, "madi_emb_lookup_q8");
}

int madi_emb_pos_q8(const madi_q8w *emb, const uint32_t *tokens, const uint32_t *pos, int m, int64_t tok_stride,
                    int tok_len, const float *pos_emb, int max_pos, float *out, void *stream) {
    if (!pos || !pos_emb || max_pos <= 0) return fail(MADI_EINVAL, "madi_emb_pos_q8: pos / pos_emb / max_pos");
    return emb_impl(emb, tokens, pos, m, tok_stride, tok_len, pos_emb, max_pos, out, stream, "madi_emb_pos_q8");
}

int madi_argmax_conf(const float *logits, int m, int vocab, uint32_t *tokens, float *conf, const uint32_t *pos,
                     int max_len, int64_t stride, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_argmax_conf: not initialised");
    if (!logits || !tokens || !pos) return fail(MADI_EINVAL, "madi_argmax_conf: null argument");
    if (m <= 0 || vocab <= 0 || max_len <= 0 || (m > 1 && stride < max_len))
        return fail(MADI_EINVAL, "madi_argmax_conf: bad shape (m=%d vocab=%d max_len=%d)", m, vocab, max_len);
    cudaError_t e = launch_argmax(logits, tokens, conf, pos, vocab, max_len, m, stride, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_argmax_conf");
}

int madi_logit_filter(float *logits, int vocab, const uint32_t *past, int past_len, const uint32_t *step,
                      uint32_t sample_begin, uint32_t no_repeat_ngram, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_logit_filter: not initialised");
    if (!logits || !past || !step || vocab <= 0 || past_len < 0) return fail(MADI_EINVAL, "madi_logit_filter: bad argument");
    cudaError_t e = launch_logit_filter(logits, past, step, sample_begin, no_repeat_ngram, vocab, past_len, 1, 0,
                                        pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_logit_filter");
}

int madi_logit_filter_rows(float *logits, int m, int vocab, const uint32_t *past, int past_len, int64_t past_stride,
                           const uint32_t *step, uint32_t sample_begin, uint32_t no_repeat_ngram, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_logit_filter_rows: not initialised");
    if (!logits || !past || !step || vocab <= 0 || past_len < 0 || m <= 0 || m > 65535 ||
        (m > 1 && past_stride < past_len))
        return fail(MADI_EINVAL, "madi_logit_filter_rows: bad argument (m=%d past_len=%d)", m, past_len);
    cudaError_t e = launch_logit_filter(logits, past, step, sample_begin, no_repeat_ngram, vocab, past_len, m,
                                        (long long)past_stride, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_logit_filter_rows");
}

int madi_suppress_rows(float *logits, int m, int vocab, const uint32_t *ids, int n, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_suppress_rows: not initialised");
    if (!logits || !ids || m <= 0 || m > 65535 || vocab <= 0 || n < 0)
        return fail(MADI_EINVAL, "madi_suppress_rows: bad argument (m=%d vocab=%d n=%d)", m, vocab, n);
    cudaError_t e = launch_suppress(logits, ids, n, vocab, m, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_suppress_rows");
}

int madi_decode_tail(float *logits, int m, int vocab, uint32_t *tokens, int64_t tok_stride, int max_len, uint32_t *pos,
                     float *conf, uint32_t sample_begin, uint32_t no_repeat_ngram, const uint32_t *suppress,
                     int n_suppress, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_decode_tail: not initialised");
    if (!logits || !tokens || !pos || (n_suppress > 0 && !suppress) || n_suppress < 0)
        return fail(MADI_EINVAL, "madi_decode_tail: null argument");
    if (m <= 0 || m > 65535 || vocab <= 0 || vocab > decode_tail_max_vocab() || max_len <= 0 ||
        (m > 1 && tok_stride < max_len))
        return fail(MADI_EINVAL, "madi_decode_tail: bad shape (m=%d vocab=%d <= %d, max_len=%d)", m, vocab,
                    decode_tail_max_vocab(), max_len);
    cudaError_t e = launch_decode_tail(logits, m, vocab, tokens, (long long)tok_stride, max_len, pos, conf, sample_begin,
                                       no_repeat_ngram, suppress, n_suppress, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_decode_tail");
}

int madi_shard_decode_tail(float *logits, int m, int n, uint32_t h0, int vocab, const uint32_t *tokens,
                           int64_t tok_stride, int max_len, const uint32_t *pos, uint32_t sample_begin,
                           uint32_t no_repeat_ngram, const uint32_t *suppress, int n_suppress, float *part,
                           void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_shard_decode_tail: not initialised");
    if (!logits || !tokens || !pos || !part || (n_suppress > 0 && !suppress) || n_suppress < 0)
        return fail(MADI_EINVAL, "madi_shard_decode_tail: null argument");
    if (m <= 0 || m > 65535 || n <= 0 || n > decode_tail_max_vocab() || vocab <= 0 || (int64_t)h0 + n > vocab ||
        max_len <= 0 || (m > 1 && tok_stride < max_len))
        return fail(MADI_EINVAL, "madi_shard_decode_tail: bad shape (m=%d n=%d <= %d, h0=%u, vocab=%d, max_len=%d)", m,
                    n, decode_tail_max_vocab(), h0, vocab, max_len);
    if (!aligned(part, 16)) return fail(MADI_EINVAL, "madi_shard_decode_tail: part must be 16-byte aligned");
    cudaError_t e = launch_shard_tail(logits, m, n, h0, vocab, tokens, (long long)tok_stride, max_len, pos, sample_begin,
                                      no_repeat_ngram, suppress, n_suppress, reinterpret_cast<float4 *>(part),
                                      pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_shard_decode_tail");
}

int madi_merge_shard_tail(const float *parts, int world, int m, uint32_t *tokens, int64_t tok_stride, int max_len,
                          uint32_t *pos, float *conf, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_merge_shard_tail: not initialised");
    if (!parts || !tokens || !pos || world <= 0 || m <= 0 || max_len <= 0 || (m > 1 && tok_stride < max_len))
        return fail(MADI_EINVAL, "madi_merge_shard_tail: bad argument (world=%d m=%d max_len=%d)", world, m, max_len);
    if (!aligned(parts, 16)) return fail(MADI_EINVAL, "madi_merge_shard_tail: parts must be 16-byte aligned");
    cudaError_t e = launch_merge_tail(reinterpret_cast<const float4 *>(parts), world, m, tokens, (long long)tok_stride,
                                      max_len, pos, conf, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_merge_shard_tail");
}

int madi_argmax_rows(const float *logits, int m, int vocab, uint32_t *tokens, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_argmax_rows: not initialised");
    if (!logits || !tokens || m <= 0 || vocab <= 0) return fail(MADI_EINVAL, "madi_argmax_rows: bad argument");
    cudaError_t e = launch_argmax(logits, tokens, nullptr, nullptr, vocab, 1, m, 1, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_argmax_rows");
}

int madi_shard_argmax(const float *logits, int m, int n, int64_t row_stride, uint32_t h0, float *vals, uint32_t *idx,
                      void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_shard_argmax: not initialised");
    if (!logits || !vals || !idx || m <= 0 || n <= 0 || row_stride < n)
        return fail(MADI_EINVAL, "madi_shard_argmax: bad argument (m=%d n=%d)", m, n);
    cudaError_t e = launch_shard_argmax(logits, (long long)row_stride, n, h0, m, vals, idx, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_shard_argmax");
}

int madi_merge_shard_argmax(const float *vals, const uint32_t *idx, int world, int m, uint32_t *tokens, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_merge_shard_argmax: not initialised");
    if (!vals || !idx || !tokens || world <= 0 || m <= 0)
        return fail(MADI_EINVAL, "madi_merge_shard_argmax: bad argument");
    cudaError_t e = launch_merge_argmax(vals, idx, world, m, tokens, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_merge_shard_argmax");
}

int madi_cross_attn(const float *q, const void *kc, const void *vc, int kv_dtype, int slots, int seqlen, int heads,
                    int kv_heads, int kv_dim, float *out, float *scores, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_cross_attn: not initialised");
    if (!q || !kc || !vc || !out || (kv_dtype != MADI_F16 && kv_dtype != MADI_F32))
        return fail(MADI_EINVAL, "madi_cross_attn: bad argument");
    if (int rc = attn_shape_ok("madi_cross_attn", 64, (uint32_t)kv_dim, (uint32_t)kv_heads, (uint32_t)heads)) return rc;
    if (slots <= 0 || slots > 65535 || seqlen <= 0 || attn_cluster_size(seqlen) == 0)
        return fail(MADI_EINVAL, "madi_cross_attn: slots %d, seqlen %d (<= %d)", slots, seqlen, 8 * kAttnMaxChunk);
    if (!aligned(q, 16) || !aligned(kc, 16) || !aligned(vc, 16) || !aligned(out, 16))
        return fail(MADI_EINVAL, "madi_cross_attn: buffers must be 16-byte aligned");
    cudaError_t e = launch_cross_attn(out, q, kc, vc, kv_dtype == MADI_F16, scores, slots, seqlen, kv_dim, kv_heads,
                                      heads, S.dev_err, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_cross_attn");
}

int madi_cross_attn_split_static(const float *q, const uint16_t *kc, const uint16_t *vc, int seqlen, int heads,
                                 int kv_heads, int kv_dim, int nsplit, float *out, float *scores, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_cross_attn_split_static: not initialised");
    if (!q || !kc || !vc || !out) return fail(MADI_EINVAL, "madi_cross_attn_split_static: null argument");
    if (int rc = attn_shape_ok("madi_cross_attn_split_static", 64, (uint32_t)kv_dim, (uint32_t)kv_heads,
                               (uint32_t)heads))
        return rc;
    if (seqlen <= 0 || nsplit <= 0 || (seqlen + nsplit - 1) / nsplit > kAttnMaxChunk)
        return fail(MADI_EINVAL, "madi_cross_attn_split_static: seqlen %d over %d splits (at most %d keys per split)",
                    seqlen, nsplit, kAttnMaxChunk);
    if ((long)heads * nsplit > kSplitStaticMax)
        return fail(MADI_EINVAL,
                    "madi_cross_attn_split_static: heads x nsplit = %ld exceeds the fixed scratch of %d partials",
                    (long)heads * nsplit, kSplitStaticMax);
    if (!aligned(q, 16) || !aligned(kc, 16) || !aligned(vc, 16) || !aligned(out, 16) || (scores && !aligned(scores, 16)))
        return fail(MADI_EINVAL, "madi_cross_attn_split_static: buffers must be 16-byte aligned");
    cudaError_t e = launch_cross_attn_split_static(out, q, kc, vc, scores, seqlen, kv_dim, kv_heads, heads, nsplit,
                                                   S.device, pick_stream(stream));
    if (e == cudaErrorInvalidDevice)
        return fail(MADI_EINVAL, "madi_cross_attn_split_static: the current device is not device %d, which "
                                 "madi_init bound", S.device);
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_cross_attn_split_static");
}

int madi_flash_attn_enc(const uint16_t *q, const uint16_t *k, const uint16_t *v, int stride, uint16_t *out,
                        int out_stride, int seq, int heads, int chunks, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_flash_attn_enc: not initialised");
    if (!q || !k || !v || !out) return fail(MADI_EINVAL, "madi_flash_attn_enc: null argument");
    if (seq <= 0 || heads <= 0 || heads > 1024 || chunks <= 0 || chunks > 65535 || stride < heads * 64 ||
        out_stride < heads * 64 || stride % 8 || out_stride % 8 || (size_t)chunks * seq >= (1ull << 31))
        return fail(MADI_EINVAL, "madi_flash_attn_enc: seq %d heads %d chunks %d stride %d out_stride %d", seq, heads,
                    chunks, stride, out_stride);
    if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16))
        return fail(MADI_EINVAL, "madi_flash_attn_enc: buffers must be 16-byte aligned");
    cudaError_t e = launch_flash_enc(reinterpret_cast<const __half *>(q), reinterpret_cast<const __half *>(k),
                                     reinterpret_cast<const __half *>(v), stride, reinterpret_cast<__half *>(out),
                                     out_stride, seq, heads, chunks, S.dev_err, pick_stream(stream));
    if (e == cudaErrorNotSupported) return fail(MADI_EUNSUPPORTED, "madi_flash_attn_enc: tensor maps unavailable");
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_flash_attn_enc");
}

int madi_self_attn(const float *q, const void *kc, const void *vc, int kv_dtype, const uint32_t *pos, int slots,
                   int heads, int kv_heads, int kv_dim, int max_tok, float *out, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_self_attn: not initialised");
    if (!q || !kc || !vc || !pos || !out || (kv_dtype != MADI_F16 && kv_dtype != MADI_F32))
        return fail(MADI_EINVAL, "madi_self_attn: bad argument");
    if (int rc = attn_shape_ok("madi_self_attn", 64, (uint32_t)kv_dim, (uint32_t)kv_heads, (uint32_t)heads)) return rc;
    if (slots <= 0 || slots > 65535 || max_tok <= 0 || max_tok > kAttnMaxTok)
        return fail(MADI_EINVAL, "madi_self_attn: slots %d, max_tok %d (<= %d)", slots, max_tok, kAttnMaxTok);
    if (!aligned(q, 16) || !aligned(kc, 16) || !aligned(vc, 16) || !aligned(out, 16))
        return fail(MADI_EINVAL, "madi_self_attn: buffers must be 16-byte aligned");
    cudaError_t e = launch_self_attn(out, q, kc, vc, kv_dtype == MADI_F16, pos, slots, kv_dim, kv_heads, heads, max_tok,
                                     S.dev_err, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_self_attn");
}

int madi_step_advance(uint32_t *pos, int m, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_step_advance: not initialised");
    if (!pos || m <= 0 || m > 32) return fail(MADI_EINVAL, "madi_step_advance: m=%d (1..32)", m);
    cudaError_t e = launch_step_advance(pos, m, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_step_advance");
}

int madi_layer_norm_f16(const float *x, uint16_t *y, const float *gamma, const float *beta, int rows, int d, float eps,
                        void *stream) {
    return res_ln_impl(const_cast<float *>(x), nullptr, nullptr, y, gamma, beta, rows, d, eps, stream,
                       "madi_layer_norm_f16");
}


/* ---- rank-to-rank all-gather over NVLink (xchg.cu) ---- */
struct madi_xchg {
    int world = 0, rank = 0;
    size_t cap = 0;
    uint8_t *own = nullptr;
    uint8_t *bases[kXchgMaxWorld] = {};
    bool opened[kXchgMaxWorld] = {};
};

int madi_xchg_create(int world, int rank, size_t cap_bytes, madi_xchg **out) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_xchg_create: not initialised");
    if (!out) return fail(MADI_EINVAL, "madi_xchg_create: null out");
    *out = nullptr;
    if (world < 1 || world > kXchgMaxWorld || rank < 0 || rank >= world)
        return fail(MADI_EINVAL, "madi_xchg_create: world %d, rank %d (1 <= world <= %d)", world, rank,
                    kXchgMaxWorld);
    if (cap_bytes == 0 || cap_bytes % 16 || cap_bytes > (64u << 20))
        return fail(MADI_EINVAL, "madi_xchg_create: cap %zu (a multiple of 16, at most 64 MiB)", cap_bytes);
    madi_xchg *x = new madi_xchg;
    x->world = world;
    x->rank = rank;
    x->cap = cap_bytes;
    const size_t n = xchg_buffer_bytes(world, cap_bytes);
    cudaError_t e = cudaMalloc(&x->own, n);
    if (e == cudaSuccess) e = cudaMemset(x->own, 0, n);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();          // zeroed before any peer maps it
    if (e != cudaSuccess) {
        if (x->own) cudaFree(x->own);
        delete x;
        return cuda_fail(e, "madi_xchg_create");
    }
    x->bases[rank] = x->own;
    x->opened[rank] = true;
    *out = x;
    return MADI_OK;
}

int madi_xchg_handle(const madi_xchg *x, void *handle64) {
    if (!x || !handle64) return fail(MADI_EINVAL, "madi_xchg_handle: null argument");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, x->own);
    if (e != cudaSuccess) return cuda_fail(e, "madi_xchg_handle");
    memcpy(handle64, &h, sizeof(h));
    return MADI_OK;
}

int madi_xchg_open(madi_xchg *x, int peer, const void *handle64) {
    if (!x || !handle64) return fail(MADI_EINVAL, "madi_xchg_open: null argument");
    if (peer < 0 || peer >= x->world || peer == x->rank || x->opened[peer])
        return fail(MADI_EINVAL, "madi_xchg_open: peer %d (world %d, rank %d)", peer, x->world, x->rank);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    void *p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "madi_xchg_open");
    x->bases[peer] = static_cast<uint8_t *>(p);
    x->opened[peer] = true;
    return MADI_OK;
}

int madi_xchg_allgather(madi_xchg *x, const void *src, size_t bytes, void *dst, void *stream) {
    if (!S.ready) return fail(MADI_ENOINIT, "madi_xchg_allgather: not initialised");
    if (!x || !src || !dst) return fail(MADI_EINVAL, "madi_xchg_allgather: null argument");
    for (int r = 0; r < x->world; ++r)
        if (!x->opened[r]) return fail(MADI_EINVAL, "madi_xchg_allgather: rank %d's buffer is not mapped", r);
    if (bytes == 0 || bytes % 16 || bytes > x->cap)
        return fail(MADI_EINVAL, "madi_xchg_allgather: %zu bytes (a multiple of 16, at most %zu)", bytes, x->cap);
    if (!aligned(src, 16) || !aligned(dst, 16)) return fail(MADI_EINVAL, "madi_xchg_allgather: misaligned buffer");
    const cudaError_t e =
        launch_xchg_allgather(x->bases, x->world, x->rank, x->cap, src, bytes, dst, S.dev_err, pick_stream(stream));
    return e == cudaSuccess ? MADI_OK : cuda_fail(e, "madi_xchg_allgather");
}

int madi_xchg_unmap(madi_xchg *x) {
    if (!x) return MADI_OK;
    for (int r = 0; r < x->world; ++r)
        if (r != x->rank && x->opened[r]) {
            cudaIpcCloseMemHandle(x->bases[r]);
            x->opened[r] = false;
            x->bases[r] = nullptr;
        }
    return MADI_OK;
}

int madi_xchg_destroy(madi_xchg *x) {
    if (!x) return MADI_OK;
    madi_xchg_unmap(x);
    if (x->own) cudaFree(x->own);
    delete x;
    return MADI_OK;
}

}  // extern "C"
