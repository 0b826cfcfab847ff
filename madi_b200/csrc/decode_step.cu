// decode_step.cu -- the GPU-resident greedy decode-step primitives around the
// Q8 projections (graph_helpers.metal:12-178, :354-388, :785-821), so a whole
// token step -- embedding, projections, vocab head, logit filter, argmax -- runs
// on the device with no host round trip between tokens and can be replayed as a
// CUDA graph (the position / step counters live in device memory).
//
//   emb_lookup_indirect_q8  out[i] = float(qs[tok*dim+i]) * float(scales[tok*nb+i/32]),
//                           tok = tokens[*pos]                             (:354-367)
//   gpu_emb_lookup_q8       same, tok = *tok_ptr                           (:370-383)
//   emb_lookup_indirect     out[i] = float(emb_f16[tok*dim+i])             (:12-23)
//   pos_embed_add_indirect  out[i] += pos_emb[*pos*dim+i]                  (:48-57)
//                           (fused into the Q8 lookup for m slots when pos_emb is given)
//   step_advance            *pos += 1                                      (:60-62)
//   argmax_no_inc           tokens[*pos] = argmax(logits)                  (:64-95)
//   argmax_conf             + conf[*pos] = 1 / sum exp(z - zmax)           (:785-821)
//   suppress_list           logits[ids[j]] = -3.4e38                       (:97-107)
//   logit_filter_indirect   special / anti-loop / n-gram / begin-window bans (:109-160)
//
// The argmax keeps the reference's reduction structure exactly -- 1024 threads,
// each scanning indices t, t+1024, ... with a strict '>', then a halving tree in
// shared memory that takes the upper slot only when strictly greater -- so ties
// resolve as the reference's do (the first index of the winning thread, the
// winning thread being the one whose 10-bit index is smallest when bit-reversed).
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"

namespace madi {
namespace {

namespace cg = cooperative_groups;

constexpr float kNeg = -3.4e38f;

// Every index that comes from device memory (a position, a token) is checked
// against the length the host derived for its buffer before it is used.
// pos_emb (optional): out[s][i] = emb + pos_emb[pos[s]][i] when pos[s] < max_pos (the
// reference's lookup followed by pos_embed_add_indirect; one f32 add, same result).
__global__ void emb_q8_kernel(float *__restrict__ out, const int8_t *__restrict__ qs, const __half *__restrict__ scales,
                              const uint32_t *__restrict__ tokens, const uint32_t *__restrict__ pos, int dim,
                              int rows, int m, long long tok_stride, long long tok_len,
                              const float *__restrict__ pos_emb, int max_pos) {
    const int s = blockIdx.y;                       // token slot
    pdl_trigger();
    pdl_wait();
    if (s >= m) return;
    const uint32_t p = pos ? pos[s] : 0u;
    const uint32_t tok = (long long)p < tok_len ? tokens[(size_t)s * tok_stride + p] : 0xffffffffu;
    const int nb = dim >> 5;
    float *o = out + (size_t)s * dim;
    if (tok >= (uint32_t)rows) {                    // out-of-range position or token: zeros, no stray read
        const float *pz = (pos_emb && p < (uint32_t)max_pos) ? pos_emb + (size_t)p * dim : nullptr;
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
            o[i] = pz ? 0.f + pz[i] : 0.f;
        return;
    }
    const int8_t *qr = qs + (size_t)tok * dim;
    const __half *sr = scales + (size_t)tok * nb;
    const float *pe = (pos_emb && p < (uint32_t)max_pos) ? pos_emb + (size_t)p * dim : nullptr;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
        const float e = (float)qr[i] * __half2float(sr[i >> 5]);
        o[i] = pe ? e + pe[i] : e;
    }
}

__global__ void emb_f16_kernel(float *__restrict__ out, const __half *__restrict__ emb,
                               const uint32_t *__restrict__ tokens, const uint32_t *__restrict__ pos, int dim, int rows,
                               long long tok_len) {
    pdl_trigger();
    pdl_wait();
    const uint32_t p = pos[0];
    const uint32_t tok = (long long)p < tok_len ? tokens[p] : 0xffffffffu;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
        out[i] = tok < (uint32_t)rows ? __half2float(emb[(size_t)tok * dim + i]) : 0.f;
}

__global__ void pos_add_kernel(float *__restrict__ out, const float *__restrict__ pos_emb,
                               const uint32_t *__restrict__ pos, int dim, int max_pos) {
    pdl_trigger();
    pdl_wait();
    const uint32_t p = pos[0];
    if (p >= (uint32_t)max_pos) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
        out[i] += pos_emb[(size_t)p * dim + i];
}

__global__ void step_advance_kernel(uint32_t *pos, int m) {
    pdl_trigger();
    pdl_wait();
    const int s = threadIdx.x;
    if (s < m) pos[s] += 1;
}

// One CTA of 1024 threads per token slot (blockIdx.x): logits row blockIdx.x.
template <bool kConf>
__global__ void __launch_bounds__(1024) argmax_kernel(const float *__restrict__ logits, uint32_t *__restrict__ tokens,
                                                      float *__restrict__ conf, const uint32_t *__restrict__ pos,
                                                      int V, int max_len, long long stride) {
    __shared__ float sv[1024];
    __shared__ uint32_t si[1024];
    const int t = threadIdx.x, s = blockIdx.x;
    pdl_trigger();
    pdl_wait();
    const float *lg = logits + (size_t)s * V;
    float lm = -INFINITY;
    uint32_t li = 0;
    // unrolled so that a thread's loads are in flight together; the compares still
    // run in index order
#pragma unroll 8
    for (int i = t; i < V; i += 1024) {
        const float v = lg[i];
        if (v > lm) { lm = v; li = (uint32_t)i; }
    }
    sv[t] = lm;
    si[t] = li;
    __syncthreads();
    for (int st = 512; st > 0; st >>= 1) {
        if (t < st && sv[t + st] > sv[t]) { sv[t] = sv[t + st]; si[t] = si[t + st]; }
        __syncthreads();
    }
    const float zmax = sv[0];
    const uint32_t amax = si[0];
    float inv_sum = 0.f;
    if constexpr (kConf) {
        __syncthreads();
        float ls = 0.f;
#pragma unroll 8
        for (int i = t; i < V; i += 1024) ls += expf(lg[i] - zmax);
        sv[t] = ls;
        __syncthreads();
        for (int st = 512; st > 0; st >>= 1) {
            if (t < st) sv[t] += sv[t + st];
            __syncthreads();
        }
        inv_sum = 1.0f / sv[0];
    }
    if (t == 0) {
        const uint32_t cur = pos ? pos[s] : 0u;
        if (cur < (uint32_t)max_len) {
            tokens[(size_t)s * stride + cur] = amax;
            if constexpr (kConf) conf[(size_t)s * stride + cur] = inv_sum;
        }
    }
}

// Row blockIdx.y of logits [rows][V].
__global__ void suppress_kernel(float *__restrict__ logits, const uint32_t *__restrict__ ids, int n, int V) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_trigger();
    pdl_wait();
    if (j >= n) return;
    const uint32_t t = ids[j];
    if (t < (uint32_t)V) logits[(size_t)blockIdx.y * V + t] = kNeg;
}

// logit_filter_indirect (graph_helpers.metal:109-160): one CTA of 256 threads per
// logits row; row r uses logits + r * V, past + r * past_stride and step_ptr[r].
__global__ void __launch_bounds__(256) logit_filter_kernel(float *__restrict__ logits,
                                                           const uint32_t *__restrict__ past,
                                                           const uint32_t *__restrict__ step_ptr, uint32_t sample_begin,
                                                           uint32_t no_repeat_ngram, int V, int past_len,
                                                           long long past_stride) {
    const uint32_t i = threadIdx.x;
    pdl_trigger();
    pdl_wait();
    logits += (size_t)blockIdx.x * V;
    past += (size_t)blockIdx.x * past_stride;
    const uint32_t step = step_ptr[blockIdx.x];
    // the history reads below stay inside past[0 .. past_len)
    const bool hist_ok = step <= (uint32_t)past_len;
    if (i == 0 && hist_ok && step >= 3 && step >= sample_begin + 3) {
        const uint32_t t1 = past[step - 1], t2 = past[step - 2], t3 = past[step - 3];
        if (t1 == t2 && t2 == t3 && t1 < (uint32_t)V) logits[t1] = kNeg;
    }
    // (sample_begin <= step keeps the window start below step even if the sums wrap)
    if (i == 0 && hist_ok && no_repeat_ngram >= 2 && step >= no_repeat_ngram && sample_begin <= step &&
        step >= sample_begin + no_repeat_ngram) {
        const uint32_t kWin = 16;
        const uint32_t n = no_repeat_ngram;
        const uint32_t suf = step - (n - 1);
        const uint32_t j0 = (step > sample_begin + kWin) ? (step - kWin) : sample_begin;
        for (uint32_t j = j0; j + n <= step; ++j) {
            bool match = true;
            for (uint32_t k = 0; k + 1 < n; ++k)
                if (past[j + k] != past[suf + k]) { match = false; break; }
            if (match) {
                const uint32_t c = past[j + n - 1];
                if (c < (uint32_t)V) logits[c] = kNeg;
            }
        }
    }
    for (uint32_t t = i + 50258; t < (uint32_t)V; t += 256) logits[t] = kNeg;
    if (step < sample_begin + 4) {
        if (i == 0 && 220 < V) logits[220] = kNeg;
        if (i == 1 && 50257 < V) logits[50257] = kNeg;
    }
}

// ---- greedy token over a column-split vocab head (one shard per GPU)
//
// The reference's tree (argmax_kernel above) prefers, among tied maxima, the
// index g whose lane g mod 1024 is smallest when its 10 bits are reversed, then
// the smallest g.  That is a total order on g, so a shard can reduce with the
// key (bitrev10(g & 1023), g) and the shards' winners merge exactly.
MADI_DEV uint64_t tie_key(uint32_t g) { return ((uint64_t)(__brev(g & 1023u) >> 22) << 32) | g; }
MADI_DEV bool better(float v, uint64_t k, float bv, uint64_t bk) { return v > bv || (v == bv && k < bk); }

// One CTA of 1024 threads per row: (max, global index) of logits[row][0..n),
// global index = h0 + local index.
__global__ void __launch_bounds__(1024) shard_argmax_kernel(const float *__restrict__ logits, long long row_stride,
                                                            int n, uint32_t h0, float *__restrict__ vals,
                                                            uint32_t *__restrict__ idx) {
    __shared__ float sv[1024];
    __shared__ uint64_t sk[1024];
    const int t = threadIdx.x, row = blockIdx.x;
    pdl_trigger();
    pdl_wait();
    const float *lg = logits + (size_t)row * row_stride;
    float bv = -INFINITY;
    uint64_t bk = ~0ull;
#pragma unroll 8
    for (int i = t; i < n; i += 1024) {
        const float v = lg[i];
        const uint64_t k = tie_key(h0 + (uint32_t)i);
        if (better(v, k, bv, bk)) { bv = v; bk = k; }
    }
    sv[t] = bv;
    sk[t] = bk;
    __syncthreads();
    for (int st = 512; st > 0; st >>= 1) {
        if (t < st && better(sv[t + st], sk[t + st], sv[t], sk[t])) { sv[t] = sv[t + st]; sk[t] = sk[t + st]; }
        __syncthreads();
    }
    if (t == 0) {
        vals[row] = sv[0];
        idx[row] = (uint32_t)sk[0];
    }
}

// tokens[row] = the best of the `world` (value, index) pairs of the row; pairs
// are rank-major: vals[r * m + row].
__global__ void merge_argmax_kernel(const float *__restrict__ vals, const uint32_t *__restrict__ idx, int world, int m,
                                    uint32_t *__restrict__ tokens) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_trigger();
    pdl_wait();
    if (row >= m) return;
    float bv = vals[row];
    uint32_t bi = idx[row];
    for (int r = 1; r < world; ++r) {
        const float v = vals[(size_t)r * m + row];
        const uint32_t i = idx[(size_t)r * m + row];
        if (better(v, tie_key(i), bv, tie_key(bi))) { bv = v; bi = i; }
    }
    tokens[row] = bi;
}

// ---- the token step's tail in one launch: step_advance, logit_filter_indirect,
// suppress_list and argmax_conf for m slots.  One cluster of kTailCtas CTAs per slot
// (blockIdx.y), CTA r owning logits [r * per, r * per + per): each CTA writes the
// filter's and the suppress list's bans that fall in its range (the same -3.4e38 the
// separate kernels write), reads its range once into registers, reduces (max,
// tie key) -- the reference's tie order as a total order, as the column-split head
// does -- and the cluster combines through rank 0's shared memory; the exp sum of
// the confidence runs over the registers against the global max.  Same tokens and
// filtered logits as the four kernels; the confidence's f32 sum runs in another
// order.
//
// kShard: the same for one column shard of the vocabulary -- the row holds global
// token ids [h0, h0 + n) of a vocabulary of V; bans apply to the ids that fall in
// the shard.  Instead of advancing pos and writing the token, CTA 0 writes the
// shard's (max value, global index, exp sum against the shard's max) to part[s],
// which merge_tail_kernel combines over the shards (with the history, position and
// suppress list every shard shares).
constexpr int kTailCtas = 8;
constexpr int kTailThr = 256;
constexpr int kTailPer = 28;                              // values per thread (n <= 8 * 256 * 28)

template <bool kShard>
__global__ void __launch_bounds__(kTailThr) decode_tail_kernel(float *__restrict__ logits, int n, uint32_t h0, int V,
                                                               uint32_t *__restrict__ tokens, long long stride,
                                                               int max_len, uint32_t *__restrict__ pos,
                                                               float *__restrict__ conf, uint32_t sample_begin,
                                                               uint32_t no_repeat_ngram,
                                                               const uint32_t *__restrict__ sup, int nsup,
                                                               float4 *__restrict__ part) {
    __shared__ float wv[kTailThr / 32];
    __shared__ uint64_t wk[kTailThr / 32];
    __shared__ float cv[kTailCtas];                       // rank 0: the CTAs' best values
    __shared__ uint64_t ck[kTailCtas];
    __shared__ float csum[kTailCtas];                     // rank 0: the CTAs' exp sums
    __shared__ float gmax;                                // every CTA: the slot's max
    __shared__ uint64_t gkey;                             // rank 0: the winner's key
    const int r = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    pdl_trigger();
    pdl_wait();
    asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
    float *lg = logits + (size_t)s * n;
    const uint32_t *past = tokens + (size_t)s * stride;
    const uint32_t step = pos[s] + 1u;                    // step_advance
    const int per = (n + kTailCtas - 1) / kTailCtas;
    const int lo = r * per, hi = min(n, lo + per);        // local columns of this CTA
    auto ban = [&](uint32_t t) {                          // t: a global token id
        if (t < (uint32_t)V && t >= h0) {
            const uint32_t c = t - h0;
            if ((int)c >= lo && (int)c < hi) lg[c] = kNeg;
        }
    };
    // logit_filter_indirect (graph_helpers.metal:109-160) with step = the advanced position
    const bool hist_ok = step <= (uint32_t)max_len;
    if (tid == 0) {
        if (hist_ok && step >= 3 && step >= sample_begin + 3) {
            const uint32_t t1 = past[step - 1], t2 = past[step - 2], t3 = past[step - 3];
            if (t1 == t2 && t2 == t3) ban(t1);
        }
        if (hist_ok && no_repeat_ngram >= 2 && step >= no_repeat_ngram && sample_begin <= step &&
            step >= sample_begin + no_repeat_ngram) {
            const uint32_t kWin = 16;
            const uint32_t nn = no_repeat_ngram;
            const uint32_t suf = step - (nn - 1);
            const uint32_t j0 = (step > sample_begin + kWin) ? (step - kWin) : sample_begin;
            for (uint32_t j = j0; j + nn <= step; ++j) {
                bool match = true;
                for (uint32_t k = 0; k + 1 < nn; ++k)
                    if (past[j + k] != past[suf + k]) { match = false; break; }
                if (match) ban(past[j + nn - 1]);
            }
        }
        if (step < sample_begin + 4) {
            ban(220u);
            ban(50257u);
        }
    }
    // ids >= 50258 (specials): local columns from max(lo, 50258 - h0)
    const int sp0 = 50258 > (int)h0 ? 50258 - (int)h0 : 0;
    for (int c = max(lo, sp0) + tid; c < hi && (uint32_t)c + h0 < (uint32_t)V; c += kTailThr) lg[c] = kNeg;
    for (int j = tid; j < nsup; j += kTailThr) ban(sup[j]);                 // suppress_list
    __syncthreads();
    float v[kTailPer];
    float bv = -INFINITY;
    uint64_t bk = ~0ull;
#pragma unroll
    for (int i = 0; i < kTailPer; ++i) {
        const int t = lo + tid + i * kTailThr;
        v[i] = t < hi ? lg[t] : -INFINITY;
    }
#pragma unroll
    for (int i = 0; i < kTailPer; ++i) {
        const int t = lo + tid + i * kTailThr;
        if (t < hi) {
            const uint64_t k = tie_key(h0 + (uint32_t)t);
            if (better(v[i], k, bv, bk)) { bv = v[i]; bk = k; }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint64_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
        if (better(ov, ok, bv, bk)) { bv = ov; bk = ok; }
    }
    if (lane == 0) { wv[warp] = bv; wk[warp] = bk; }
    __syncthreads();
    cg::cluster_group cluster = cg::this_cluster();
    asm volatile("barrier.cluster.wait;" ::: "memory");
    if (tid == 0) {
        for (int w = 1; w < kTailThr / 32; ++w)
            if (better(wv[w], wk[w], bv, bk)) { bv = wv[w]; bk = wk[w]; }
        *cluster.map_shared_rank(&cv[r], 0) = bv;
        *cluster.map_shared_rank(&ck[r], 0) = bk;
    }
    cluster.sync();
    if (r == 0 && tid < kTailCtas) {
        // rank 0: the slot's max, to every CTA
        float gv = cv[0];
        uint64_t gk = ck[0];
        for (int c = 1; c < kTailCtas; ++c)
            if (better(cv[c], ck[c], gv, gk)) { gv = cv[c]; gk = ck[c]; }
        *cluster.map_shared_rank(&gmax, tid) = gv;
        if (tid == 0) gkey = gk;
    }
    cluster.sync();
    const float zmax = gmax;
    float ls = 0.f;
#pragma unroll
    for (int i = 0; i < kTailPer; ++i)
        if (lo + tid + i * kTailThr < hi) ls += expf(v[i] - zmax);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    if (lane == 0) wv[warp] = ls;
    __syncthreads();
    if (tid == 0) {
        float cs = 0.f;
        for (int w = 0; w < kTailThr / 32; ++w) cs += wv[w];
        *cluster.map_shared_rank(&csum[r], 0) = cs;
    }
    cluster.sync();
    if (r == 0 && tid == 0) {
        float tot = 0.f;
        for (int c = 0; c < kTailCtas; ++c) tot += csum[c];
        if constexpr (kShard) {
            part[s] = make_float4(zmax, __uint_as_float((uint32_t)gkey), tot, 0.f);
        } else {
            pos[s] = step;
            if (step < (uint32_t)max_len) {
                tokens[(size_t)s * stride + step] = (uint32_t)gkey;
                if (conf) conf[(size_t)s * stride + step] = 1.0f / tot;
            }
        }
    }
}

// Combines the shards' (max, index, exp sum) of every row -- part[r * m + row], shard
// (rank) major -- into the greedy token: the best (max, tie key), the confidence
// 1 / sum_r sum_r * exp(max_r - max), then step_advance and the token / confidence
// writes of decode_tail_kernel.  One thread per row.
__global__ void merge_tail_kernel(const float4 *__restrict__ part, int world, int m, uint32_t *__restrict__ tokens,
                                  long long stride, int max_len, uint32_t *__restrict__ pos, float *__restrict__ conf) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_trigger();
    pdl_wait();
    if (row >= m) return;
    float bv = -INFINITY;
    uint32_t bi = 0;
    uint64_t bk = ~0ull;
    for (int r = 0; r < world; ++r) {
        const float4 p = part[(size_t)r * m + row];
        const uint32_t i = __float_as_uint(p.y);
        if (better(p.x, tie_key(i), bv, bk)) { bv = p.x; bi = i; bk = tie_key(i); }
    }
    float tot = 0.f;
    for (int r = 0; r < world; ++r) {
        const float4 p = part[(size_t)r * m + row];
        if (p.z > 0.f) tot += p.z * expf(p.x - bv);
    }
    const uint32_t step = pos[row] + 1u;
    pos[row] = step;
    if (step < (uint32_t)max_len) {
        tokens[(size_t)row * stride + step] = bi;
        if (conf) conf[(size_t)row * stride + step] = 1.0f / tot;
    }
}

}  // namespace

cudaError_t launch_emb_q8(float *out, const int8_t *qs, const __half *scales, const uint32_t *tokens,
                          const uint32_t *pos, int dim, int rows, int m, long long tok_stride, long long tok_len,
                          const float *pos_emb, int max_pos, cudaStream_t st) {
    return launch_k(emb_q8_kernel, dim3((dim + 255) / 256, m), 256, 0, st, 1, out, qs, scales, tokens, pos, dim, rows, m,
                    tok_stride, tok_len, pos_emb, max_pos);
}

cudaError_t launch_emb_f16(float *out, const __half *emb, const uint32_t *tokens, const uint32_t *pos, int dim,
                           int rows, long long tok_len, cudaStream_t st) {
    return launch_k(emb_f16_kernel, (dim + 255) / 256, 256, 0, st, 1, out, emb, tokens, pos, dim, rows, tok_len);
}

cudaError_t launch_pos_add(float *out, const float *pos_emb, const uint32_t *pos, int dim, int max_pos,
                           cudaStream_t st) {
    return launch_k(pos_add_kernel, (dim + 255) / 256, 256, 0, st, 1, out, pos_emb, pos, dim, max_pos);
}

cudaError_t launch_step_advance(uint32_t *pos, int m, cudaStream_t st) {
    return launch_k(step_advance_kernel, 1, 32, 0, st, 1, pos, m);
}

cudaError_t launch_argmax(const float *logits, uint32_t *tokens, float *conf, const uint32_t *pos, int V,
                          int max_len, int m, long long stride, cudaStream_t st) {
    return conf ? launch_k(argmax_kernel<true>, m, 1024, 0, st, 1, logits, tokens, conf, pos, V, max_len, stride)
                : launch_k(argmax_kernel<false>, m, 1024, 0, st, 1, logits, tokens, static_cast<float *>(nullptr), pos,
                           V, max_len, stride);
}

cudaError_t launch_suppress(float *logits, const uint32_t *ids, int n, int V, int rows, cudaStream_t st) {
    return n > 0 ? launch_k(suppress_kernel, dim3((n + 255) / 256, rows), 256, 0, st, 1, logits, ids, n, V)
                 : cudaSuccess;
}

cudaError_t launch_logit_filter(float *logits, const uint32_t *past, const uint32_t *step_ptr, uint32_t sample_begin,
                                uint32_t no_repeat_ngram, int V, int past_len, int rows, long long past_stride,
                                cudaStream_t st) {
    return launch_k(logit_filter_kernel, rows, 256, 0, st, 1, logits, past, step_ptr, sample_begin, no_repeat_ngram, V,
                    past_len, past_stride);
}

int decode_tail_max_vocab() { return kTailCtas * kTailThr * kTailPer; }

cudaError_t launch_decode_tail(float *logits, int m, int V, uint32_t *tokens, long long stride, int max_len,
                               uint32_t *pos, float *conf, uint32_t sample_begin, uint32_t no_repeat_ngram,
                               const uint32_t *sup, int nsup, cudaStream_t st) {
    return launch_k(decode_tail_kernel<false>, dim3(kTailCtas, m), kTailThr, 0, st, kTailCtas, logits, V, 0u, V,
                    tokens, stride, max_len, pos, conf, sample_begin, no_repeat_ngram, sup, nsup,
                    static_cast<float4 *>(nullptr));
}

cudaError_t launch_shard_tail(float *logits, int m, int n, uint32_t h0, int V, const uint32_t *tokens,
                              long long stride, int max_len, const uint32_t *pos, uint32_t sample_begin,
                              uint32_t no_repeat_ngram, const uint32_t *sup, int nsup, float4 *part, cudaStream_t st) {
    return launch_k(decode_tail_kernel<true>, dim3(kTailCtas, m), kTailThr, 0, st, kTailCtas, logits, n, h0, V,
                    const_cast<uint32_t *>(tokens), stride, max_len, const_cast<uint32_t *>(pos),
                    static_cast<float *>(nullptr), sample_begin, no_repeat_ngram, sup, nsup, part);
}

cudaError_t launch_merge_tail(const float4 *part, int world, int m, uint32_t *tokens, long long stride, int max_len,
                              uint32_t *pos, float *conf, cudaStream_t st) {
    return launch_k(merge_tail_kernel, (m + 127) / 128, 128, 0, st, 1, part, world, m, tokens, stride, max_len, pos,
                    conf);
}

cudaError_t launch_shard_argmax(const float *logits, long long row_stride, int n, uint32_t h0, int m, float *vals,
                                uint32_t *idx, cudaStream_t st) {
    return launch_k(shard_argmax_kernel, m, 1024, 0, st, 1, logits, row_stride, n, h0, vals, idx);
}

cudaError_t launch_merge_argmax(const float *vals, const uint32_t *idx, int world, int m, uint32_t *tokens,
                                cudaStream_t st) {
    return launch_k(merge_argmax_kernel, (m + 127) / 128, 128, 0, st, 1, vals, idx, world, m, tokens);
}

}  // namespace madi
