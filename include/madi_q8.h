/*
 * madi_q8.h -- C ABI of the B200 (sm_100a) Q8_0 linear layer.
 *
 * Drop-in for the Q8 path of companyjupiter/madi's engine operator API
 * (engine/metal/metal_backend.h + metal_backend.zig).  The reference's Zig host
 * binds that header with `extern fn` declarations (metal_backend.zig:12-32); a
 * Zig caller binds this one the same way or through @cImport.  Each entry point
 * below names the reference interface it replaces.
 *
 * Conventions (same as the reference):
 *   - Q8_0 weight: qs int8 [N][K] row-major (K contiguous) + scales f16 [N][K/32];
 *     deq(n,k) = qs[n*K+k] * scales[n*(K/32) + k/32]   (q8_gemm.metal:2-3).
 *     K must be a multiple of 32.
 *   - Every pointer is a caller-owned DEVICE pointer unless stated; the library
 *     never frees caller buffers (metal_backend.m:336-361 ownership rule).
 *   - Every int-returning entry returns MADI_OK (0) on success and a negative
 *     MADI_E* code on failure, so the reference's `!= 0 -> error` checks
 *     (metal_backend.zig:34-41) keep working.  Argument checks happen before
 *     any launch.
 *   - Not thread-safe per process except madi_alloc/madi_free (the reference's
 *     g_alloc_mutex rule, metal_backend.m:99).  One device per process.
 */
#ifndef MADI_Q8_H
#define MADI_Q8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define MADI_OK             0
#define MADI_ERR           -1   /* generic failure (the reference's -1) */
#define MADI_EINVAL        -2   /* bad argument: shape, alignment, null, dtype */
#define MADI_ENOTFOUND     -3   /* unknown kernel name */
#define MADI_ECUDA         -4   /* CUDA runtime error (see madi_last_error) */
#define MADI_ETIMEDOUT     -5   /* madi_sync timed out; work still pending */
#define MADI_ENOINIT       -6   /* madi_init not called / failed */
#define MADI_EDEVICE       -7   /* a kernel's bounded wait expired (device error flag) */
#define MADI_EUNSUPPORTED  -8   /* device is not sm_100 / feature unavailable */
#define MADI_EBUSY         -9   /* command buffer already open / not open */

/* ---- element types ------------------------------------------------------ */
#define MADI_F32  0
#define MADI_F16  1
/* Activations stored as f32 and rounded to f16 when the kernel loads them, as the
 * reference's batched decode (decodeBlockBatched, decoder.zig:337-341) converts its
 * f32 activations to f16 before the projection; madi_q8_linear's streaming path only. */
#define MADI_F32_AS_F16  2

/* ---- epilogues (bias / GELU / residual flags of the reference kernels) ---- */
#define MADI_EPI_NONE       0   /* y = acc                       gemv_q8, m4_gemm_nn, logit_gemv_q8 */
#define MADI_EPI_BIAS       1   /* y = acc + b                   gemv_q8_bias, m4_gemm_bias */
#define MADI_EPI_BIAS_GELU  2   /* y = gelu_erf(acc + b)         gemv_q8_bias_gelu, m4_gemm_bias_gelu */
#define MADI_EPI_BIAS_RES   3   /* y = r + acc + b               gemv_q8_bias_res (r may alias y),
                                   encoder residual of bias_res_ln_f16 (encoder_ops.metal:343) */

/* Q8_0 weight handle.  Replaces `Q8 = struct { qs: [*]i8, scales: [*]f16 }`
 * (encoder.zig:20-21, decoder.zig:22); carries its shape. */
typedef struct madi_q8w {
    const int8_t   *qs;       /* [n][k] */
    const uint16_t *scales;   /* [n][k/32] f16 bit patterns */
    int32_t n;                /* out features (rows) */
    int32_t k;                /* in features, multiple of 32 */
} madi_q8w;

/* ======================= lifecycle / memory =============================== */

/* mtl_init (metal_backend.h:15): bind `device`, create the stream, check sm_100. */
int   madi_init(int device);
/* mtl_cleanup (metal_backend.h:16): free library-owned state (never user buffers). */
void  madi_cleanup(void);
/* mtl_alloc / mtl_free (metal_backend.h:21-22): device memory, registered so
 * madi_dispatch can bind base or interior pointers.  256-byte aligned. */
void *madi_alloc(size_t size);
void  madi_free(void *ptr);
/* mtl_upload / mtl_download (metal_backend.h:30-31): host <-> device copies
 * (synchronous with respect to the library stream). */
int   madi_upload(void *dst_device, const void *src_host, size_t size);
int   madi_download(void *dst_host, const void *src_device, size_t size);

/* ======================= kernels by name ================================== */

/* mtl_get_function (metal_backend.h:47).  Accepted names and argument orders
 * are the reference kernels' buffer orders:
 *   gemv_q8            (out f32, qs, scales, x f32, N u32, K u32)           graph_helpers.metal:390
 *   gemv_q8_bias       (out, qs, scales, x, bias f32, N, K)                 graph_helpers.metal:424
 *   gemv_q8_bias_gelu  (out, qs, scales, x, bias, N, K)                     graph_helpers.metal:475
 *   gemv_q8_bias_res   (out, qs, scales, x, bias, N, K)   out += acc+bias   graph_helpers.metal:498
 *   gemv_q8_qkv        (q_out, qs, scales, x, qb, vb, kc, vc, pos_ptr u32*, D u32)  graph_helpers.metal:527
 *   logit_gemv_q8      (logits, qs, scales, x, vocab u32, dim u32)          graph_helpers.metal:320
 *   dequant_q8_f16     (out f16 [K][N], qs, scales, N, K)                   q8_gemm.metal:12
 *   mul_mm_q8          (C f16, A f16, qs, scales, M, N, K)                  q8_gemm.metal:29
 *   m4_gemm_q8tg       (A f16, Wq, scales, C f16, bias f32, M, N, K, act_gelu u32)  m4_gemm.metal:196
 *   m4_gemm_q8_bias_gelu (same arguments as m4_gemm_q8tg)                   m4_gemm.metal:131
 *   bias_res_ln_f16    (X f32, MO f16, bias f32, Y f16, gamma f32, beta f32, D u32, eps f32)
 *                      rows = grid_x, as the reference's grid                encoder_ops.metal:333
 *   layer_norm_f16     (X f32, Y f16, gamma f32, beta f32, D u32, eps f32)
 *                      rows = grid_x                                        encoder_ops.metal:305
 *   bias_res_ln        (X f32, MO f32, bias f32, Y f32, gamma, beta, D, eps), rows = grid_x
 *                                                                           encoder_ops.metal:69
 *   layer_norm         (X f32, Y f32, gamma, beta, D, eps), rows = grid_x   encoder_ops.metal:14
 * GPU-resident decode-step primitives (VOCAB = 51866 as in the reference; the
 * lengths of buffers read through device-held indices are taken from their
 * allocations, so out-of-range positions / tokens never read out of bounds):
 *   emb_lookup_indirect_q8 (out f32, qs, scales, tokens u32*, pos_ptr u32*, dim)  graph_helpers.metal:354
 *   gpu_emb_lookup_q8      (out f32, qs, scales, tok_ptr u32*, dim)           graph_helpers.metal:370
 *   emb_lookup_indirect    (out f32, emb f16, tokens, pos_ptr, dim)           graph_helpers.metal:12
 *   pos_embed_add_indirect (out f32, pos_emb f32, pos_ptr, dim)               graph_helpers.metal:48
 *   step_advance           (pos_ptr)                                          graph_helpers.metal:60
 *   argmax_no_inc          (logits, tokens, pos_ptr, max_len u32)             graph_helpers.metal:64
 *   argmax_conf            (logits, tokens, conf f32*, pos_ptr, max_len)      graph_helpers.metal:785
 *   suppress_list          (logits, ids u32*, n u32)                          graph_helpers.metal:97
 *   logit_filter_indirect  (logits, past_tokens, num_suppress u32, step_ptr, sample_begin u32,
 *                           no_repeat_ngram u32)                              graph_helpers.metal:109
 * Decoder attention (head_dim 64; extents taken from the allocations):
 *   gpu_attention          (out, q, kc f32, vc f32, pos_ptr, hdd, kvd, nkv, nh) decoder_ops.metal:85
 *   flash_cross_attn       (out, q, kc f32, vc f32, seqlen, hdd, kvd, nkv, nh)  decoder_ops.metal:194
 *   flash_cross_attn_f16kv (out, q, kc f16, vc f16, seqlen, hdd, kvd, nkv, nh, sc_out f32*,
 *                           write_sc u32)                                      decoder_ops.metal:254
 *   flash_cross_attn_f16kv_batched (same first nine; slots = grid_x / nh)      decoder_ops.metal:466
 *   flash_cross_attn_split (part f32*, q, kc, vc, seqlen, hdd, kvd, nkv, nh, nsplit, sc_raw, write_sc)
 *                                                                              decoder_ops.metal:338
 *   flash_cross_attn_reduce (out, part, hdd, nsplit, sc_out, seqlen, write_sc), heads = grid_x
 *                                                                              decoder_ops.metal:416
 *   m4_flash_enc           (out, q, k, v, seq_len, nh): packed [seq][nh*64] f16 m4_gemm.metal:268
 * On success *out_id holds a handle for madi_dispatch. */
int   madi_get_function(const char *name, int *out_id);

/* mtl_dispatch (metal_backend.h:53-56): `args[i]` points at the i-th argument
 * value and `arg_sizes[i]` is its size -- the cuLaunchKernel kernelParams
 * convention the reference uses.  Pointer arguments must be device pointers
 * (madi_alloc'd, base or interior, or any other device allocation).  The
 * grid/block values are accepted for compatibility and ignored -- each B200
 * kernel picks its own launch shape -- except grid_x of the two LayerNorm
 * kernels, which is their row count as in the reference.  Inside begin/commit the launch is
 * recorded into the open command buffer, otherwise it is enqueued at once. */
int   madi_dispatch(int func_id,
                    uint32_t grid_x, uint32_t grid_y, uint32_t grid_z,
                    uint32_t block_x, uint32_t block_y, uint32_t block_z,
                    const void **args, const size_t *arg_sizes, int n_args);

/* ======================= command buffers / sync =========================== */

/* mtl_begin_command_buffer / mtl_commit_command_buffer (metal_backend.h:65-68):
 * begin opens a CUDA stream capture; commit closes it into a CUDA graph and
 * launches it (the graph executable is reused when the recorded work has the
 * same shape).  Returns MADI_EBUSY on mismatched begin/commit. */
int   madi_begin_command_buffer(void);
int   madi_commit_command_buffer(void);
/* mtl_flush (metal_backend.h:59): no-op (launches are already enqueued). */
void  madi_flush(void);
/* mtl_sync (metal_backend.h:62), with a bound: waits up to timeout_ms (<0 =
 * no bound) for all enqueued work; MADI_ETIMEDOUT instead of hanging,
 * MADI_EDEVICE if a kernel reported an expired wait, MADI_ECUDA on a CUDA error. */
int   madi_sync(int timeout_ms);

/* Stream binding (no reference counterpart: the reference owns one queue).
 * stream = a cudaStream_t; NULL restores the library stream. */
int   madi_set_stream(void *cuda_stream);
void *madi_get_stream(void);

/* ======================= diagnostics ====================================== */
/* Last error message of this thread (never NULL). */
const char *madi_last_error(void);
/* mtl_set_verbose (metal_backend.h:91). */
void  madi_set_verbose(int v);
/* mtl_dump_profile (metal_backend.h:81): with MADI_PROFILE=1 each dispatch is
 * timed with CUDA events; this writes an nsys cuda_gpu_kern_sum-style table
 * (out_path NULL -> stdout). */
void  madi_dump_profile(const char *out_path);
/* Number of streaming multiprocessors of the bound device (0 before init). */
int   madi_num_sms(void);

/* ======================= typed Q8 API ===================================== */

/* Y[m][n] = epi( sum_k X[m][k] * deq(n,k) ).  Replaces the reference's
 * per-projection pairs (kDeq + m4_gemm_bias / _bias_gelu / _nn, encoder.zig:262-304;
 * the gemv_q8* family, decoder.zig:155-200; the batched f16 projection,
 * decoder.zig:337-341).  One call, no dequant scratch:
 *   m > 16 (or 9..16 when K % 256 != 0): tcgen05 tensor-core GEMM, X f16, Y f16,
 *           residual f16 (Y f32 is accepted with MADI_EPI_NONE: unrounded f32
 *           sums, e.g. the logits of a vocab head over many token slots; and with
 *           MADI_EPI_BIAS_RES and an f32 residual: Y = (residual + half(acc)) +
 *           bias, the encoder's f32 residual stream updated in the epilogue -- the
 *           add of bias_res_ln_f16, encoder_ops.metal:343-347, on the f16 projection
 *           output; residual may be Y); f16 dequantised weights, f32 accumulation.
 *   m <= 16: bandwidth-bound skinny GEMM, X f32, f16 or MADI_F32_AS_F16, Y f32 or f16,
 *           residual with Y's type and may alias Y; f32 semantics
 *           (exact int8 weights, per-block f32 scale).  (The reference's GEMV
 *           family takes one token; its batched decode takes up to 8 slots.)
 * bias: f32 or f16 per bias_dtype, required unless epi == MADI_EPI_NONE.
 * x, y, residual: row-major, rows of k (x) / n (y, residual) elements, 16-byte
 * aligned base pointers.  stream: cudaStream_t or NULL (library stream). */
int madi_q8_linear(const madi_q8w *w, const void *x, int x_dtype, int m,
                   const void *bias, int bias_dtype, int epi,
                   const void *residual, void *y, int y_dtype, void *stream);

/* Decoder self-attention QKV projection with the KV-cache store fused
 * (gemv_q8_qkv, graph_helpers.metal:527-567) for m <= 16 token slots, f32 x.
 * w: stacked [3D][D]; x f32 [m][D].  For slot s: q_out[s][0..D) = q + qb;
 * kc[s*cache_stride + pos[s]*D + j] = k_j;  vc[...] = v_j + vb[j].
 * pos: device u32 [m] (read on the device, so a graph can replay it);
 * cache_stride: elements between slots' caches (ignored for m == 1). */
int madi_q8_qkv(const madi_q8w *w, const float *x, int m,
                const float *qb, const float *vb, float *q_out,
                float *kc, float *vc, const uint32_t *pos, int64_t cache_stride,
                void *stream);

/* madi_q8_qkv with an activation type (same reference kernel): x_dtype MADI_F32;
 * MADI_F32_AS_F16 -- x f32 rounded to f16 as it is loaded, as the reference's batched
 * decode (decodeBlockBatched, decoder.zig:337-341) rounds its activations; or MADI_F16
 * -- x already f16 [m][D] (e.g. from madi_layer_norm_y16), the same values. */
int madi_q8_qkv_ex(const madi_q8w *w, const void *x, int x_dtype, int m,
                   const float *qb, const float *vb, float *q_out,
                   float *kc, float *vc, const uint32_t *pos, int64_t cache_stride,
                   void *stream);

/* dequant_q8_f16 (q8_gemm.metal:12-27): out f16 [K][N] = half(q*s), transposed. */
int madi_q8_dequant_f16(const madi_q8w *w, uint16_t *out, void *stream);

/* quantInto (transcribe.zig:309-327) on the device: w f16 [rows][dim] ->
 * qs int8 [rows][dim], scales f16 [rows][dim/32].  Bit-identical to the
 * reference's quantiser (round half away from zero on w * (1/s_f32)). */
int madi_q8_quantize_f16(const uint16_t *w, int rows, int dim,
                         int8_t *qs, uint16_t *scales, void *stream);

/* ======================= residual + LayerNorm beside the linear ============ */

/* bias_res_ln_f16 (encoder_ops.metal:333-364), the encoder's step after the
 * out-projection / fc2: for each of `rows` rows of width d,
 *   x[r][i] += float(mo[r][i]) + bias[i]      (f32 residual stream, in place)
 *   y[r][i]  = half((x[r][i] - mean) * rsqrt(var + eps) * gamma[i] + beta[i])
 * with mean and var over the updated row (two passes).  x is updated exactly as
 * the reference does ((x + mo) + bias in f32).  128 <= d <= 2048, d % 128 == 0;
 * f32 buffers 16-byte and f16 buffers 8-byte aligned. */
int madi_bias_res_ln_f16(float *x, const uint16_t *mo, const float *bias, uint16_t *y,
                         const float *gamma, const float *beta, int rows, int d, float eps,
                         void *stream);

/* layer_norm_f16 (encoder_ops.metal:305-331): y = half(LN(x) * gamma + beta),
 * x f32 [rows][d] unchanged.  Same shape and alignment rules. */
int madi_layer_norm_f16(const float *x, uint16_t *y, const float *gamma, const float *beta,
                        int rows, int d, float eps, void *stream);

/* bias_res_ln / layer_norm (encoder_ops.metal:14-120), the decoder's f32 forms:
 * x f32 [rows][d] += mo f32 + bias (in place), y f32 = LN(x) * gamma + beta.
 * Same shape and alignment rules as the f16 forms (f32 rows 16-byte aligned). */
int madi_bias_res_ln(float *x, const float *mo, const float *bias, float *y, const float *gamma, const float *beta,
                     int rows, int d, float eps, void *stream);
int madi_layer_norm(const float *x, float *y, const float *gamma, const float *beta, int rows, int d, float eps,
                    void *stream);

/* The same two with y written as f16 (round to nearest): the LayerNorm and the
 * f32 -> f16 conversion the reference's batched decode applies to a projection's
 * input (decodeBlockBatched, decoder.zig:337-341) in one pass -- bit-equal to
 * madi_bias_res_ln / madi_layer_norm followed by that rounding.  No single
 * reference kernel; y rows 8-byte aligned. */
int madi_bias_res_ln_y16(float *x, const float *mo, const float *bias, uint16_t *y, const float *gamma,
                         const float *beta, int rows, int d, float eps, void *stream);
int madi_layer_norm_y16(const float *x, uint16_t *y, const float *gamma, const float *beta, int rows, int d,
                        float eps, void *stream);

/* ======================= GPU-resident greedy decode step ==================== */

/* Q8 token-embedding lookup for m slots (emb_lookup_indirect_q8 / gpu_emb_lookup_q8,
 * graph_helpers.metal:354-383): out[s][i] = float(qs[tok][i]) * float(scales[tok][i/32]),
 * tok = tokens[s*tok_stride + pos[s]] (pos != NULL) or tokens[s] (pos == NULL).
 * A position >= tok_len or a token >= emb->n gives a zero row.  out f32 [m][emb->k]. */
int madi_emb_lookup_q8(const madi_q8w *emb, const uint32_t *tokens, const uint32_t *pos, int m,
                       int64_t tok_stride, int tok_len, float *out, void *stream);

/* madi_emb_lookup_q8 followed by pos_embed_add_indirect (graph_helpers.metal:48-57)
 * for m slots in one launch: out[s][i] = emb(tok)[i] + pos_emb[pos[s]][i] when
 * pos[s] < max_pos (else the embedding alone).  pos_emb f32 [max_pos][emb->k]. */
int madi_emb_pos_q8(const madi_q8w *emb, const uint32_t *tokens, const uint32_t *pos, int m,
                    int64_t tok_stride, int tok_len, const float *pos_emb, int max_pos, float *out,
                    void *stream);

/* Greedy token per slot (argmax_conf, graph_helpers.metal:785-821): for slot s,
 * tokens[s*stride + pos[s]] = argmax(logits[s][0..vocab)) and, if conf != NULL,
 * conf[s*stride + pos[s]] = 1 / sum_i exp(logits[s][i] - max), when pos[s] < max_len.
 * Ties resolve exactly as the reference's 1024-thread reduction does. */
int madi_argmax_conf(const float *logits, int m, int vocab, uint32_t *tokens, float *conf,
                     const uint32_t *pos, int max_len, int64_t stride, void *stream);

/* logit_filter_indirect (graph_helpers.metal:109-160) on one logits row: bans
 * tokens >= 50258, a token repeated three times, a repeated n-gram completion
 * (no_repeat_ngram >= 2, last 16 tokens), and space / EOT during the first four
 * generated steps; *step is read on the device; past holds past_len tokens. */
int madi_logit_filter(float *logits, int vocab, const uint32_t *past, int past_len,
                      const uint32_t *step, uint32_t sample_begin, uint32_t no_repeat_ngram,
                      void *stream);

/* madi_logit_filter on m rows in one launch: row r filters logits + r*vocab with
 * history past + r*past_stride (past_len tokens) and step[r]. */
int madi_logit_filter_rows(float *logits, int m, int vocab, const uint32_t *past, int past_len,
                           int64_t past_stride, const uint32_t *step, uint32_t sample_begin,
                           uint32_t no_repeat_ngram, void *stream);

/* ============================ decoder attention ============================== */

/* Cross-attention of one query token per slot over `seqlen` encoder positions
 * (flash_cross_attn / _f16kv / _f16kv_batched, decoder_ops.metal:191-531):
 * q f32 [slots][heads*64]; kc, vc [slots][seqlen][kv_dim] (MADI_F16 or MADI_F32);
 * head h reads kv head h * kv_heads / heads; out f32 [slots][heads*64];
 * scores (nullable) f32 [slots][heads][seqlen] normalised.  head_dim 64,
 * seqlen <= 2048; one thread-block cluster per (slot, head). */
int madi_cross_attn(const float *q, const void *kc, const void *vc, int kv_dtype, int slots, int seqlen, int heads,
                    int kv_heads, int kv_dim, float *out, float *scores, void *stream);

/* No counterpart in the reference.  Cross-attention of one query token over `seqlen`
 * f16 keys in the two-pass split form (the arithmetic of flash_cross_attn_split +
 * flash_cross_attn_reduce, in one call) for callers that cannot allocate device
 * memory: a decode loop driven from a real-time audio callback, where cudaMalloc and
 * cudaFree may block or synchronise the whole device, or a host application that
 * gives this library a fixed memory budget at start-up and no allocator afterwards.
 * The split partials, which the reference's form keeps in a buffer the caller
 * allocates, live here in a fixed array inside the library: it allocates nothing.
 * q f32 [heads*64]; kc, vc f16 [seqlen][kv_dim]; out f32 [heads*64]; scores f32
 * [heads][seqlen] (normalised) or NULL; at most 256 keys per split.  Limit: heads x
 * nsplit <= 2048 (the array holds 2048 x 66 floats, 528 KB, on every GPU that loads
 * the library, until the process exits); larger requests return MADI_EINVAL, and so
 * does a call while another device than the one madi_init bound is current.  The
 * first call on a device (and after its context was re-created) looks up the
 * array's device address; make that first call before any stream capture.  Every
 * call shares the one array: calls whose kernels overlap on the GPU (different
 * streams, or other threads) race on it. */
int madi_cross_attn_split_static(const float *q, const uint16_t *kc, const uint16_t *vc, int seqlen,
                                 int heads, int kv_heads, int kv_dim, int nsplit, float *out,
                                 float *scores, void *stream);

/* Encoder self-attention, bidirectional (m4_flash_enc, m4_gemm.metal:255-407) on
 * the tensor cores: for each of `chunks` sequences of `seq` rows and each head h,
 * out[t][h*64..] = softmax(Q K^T * 0.125) V over the sequence, P rounded to f16,
 * f32 accumulation, out = half(O / (l + 1e-6)).  q / k / v / out: f16 rows of
 * `stride` / `out_stride` elements (multiples of 8; the packed [q | k | v] rows of
 * the QKV projection work with k = q + heads*64, v = q + 2*heads*64), chunk c at
 * rows c*seq .. c*seq + seq - 1; head_dim 64; 16-byte aligned. */
int madi_flash_attn_enc(const uint16_t *q, const uint16_t *k, const uint16_t *v, int stride, uint16_t *out,
                        int out_stride, int seq, int heads, int chunks, void *stream);

/* Self-attention of one query token per slot over its cache rows 0..pos[slot]
 * (gpu_attention, decoder_ops.metal:81-149): kc, vc [slots][max_tok][kv_dim]
 * (MADI_F32 as the reference, or MADI_F16); pos u32 [slots] on the device
 * (positions >= max_tok attend max_tok rows); max_tok <= 512. */
int madi_self_attn(const float *q, const void *kc, const void *vc, int kv_dtype, const uint32_t *pos, int slots,
                   int heads, int kv_heads, int kv_dim, int max_tok, float *out, void *stream);

/* The tail of a greedy token step for m slots in one launch, equal to madi_step_advance,
 * madi_logit_filter_rows (history tokens[s], step = the advanced pos[s]),
 * madi_suppress_rows (ids, may be NULL with n_suppress 0) and madi_argmax_conf in turn:
 * pos[s] += 1; row s of logits [m][vocab] filtered in place; tokens[s][pos[s]] =
 * its greedy token (the reference's tie order) and conf[s][pos[s]] (conf may be
 * NULL) = 1 / sum exp(z - zmax) when pos[s] < max_len.  The confidence's f32 sum runs
 * in another order than argmax_conf's (within 1e-5 relative).  vocab <= 57344. */
int madi_decode_tail(float *logits, int m, int vocab, uint32_t *tokens, int64_t tok_stride,
                     int max_len, uint32_t *pos, float *conf, uint32_t sample_begin,
                     uint32_t no_repeat_ngram, const uint32_t *suppress, int n_suppress,
                     void *stream);

/* suppress_list (graph_helpers.metal:97-107) on m logit rows in one launch:
 * logits[r][ids[j]] = -3.4e38 for every id < vocab (ids u32 [n], on the device). */
int madi_suppress_rows(float *logits, int m, int vocab, const uint32_t *ids, int n, void *stream);

/* Greedy token of each of m full logit rows (tokens[s], no position), the
 * reference's argmax including its tie order (graph_helpers.metal:64-95). */
int madi_argmax_rows(const float *logits, int m, int vocab, uint32_t *tokens, void *stream);

/* Column-split vocab head (one shard per GPU; no reference counterpart: the
 * reference engine runs the head on one device).  madi_shard_argmax reduces
 * each of m rows of this shard's logits (n columns, global index h0 + column)
 * to a (value, global index) pair, ties ordered as the reference's argmax
 * orders them; madi_merge_shard_argmax takes the all-gathered pairs (rank-major,
 * vals[r * m + row]) and writes the greedy token of each row.  Together they give
 * the same tokens as madi_argmax_rows over the gathered full rows. */
int madi_shard_argmax(const float *logits, int m, int n, int64_t row_stride, uint32_t h0, float *vals, uint32_t *idx,
                      void *stream);
int madi_merge_shard_argmax(const float *vals, const uint32_t *idx, int world, int m, uint32_t *tokens, void *stream);

/* madi_decode_tail over a column-split vocab head (no reference counterpart: the
 * reference runs the head on one device).  Each rank holds logits [m][n] for the
 * global token ids [h0, h0 + n) of a `vocab`-token vocabulary, for ALL m token
 * rows of the job, and the same token history / positions / suppress list for
 * them (tokens [m][tok_stride], pos [m], read only here).  madi_shard_decode_tail
 * applies the filter and suppress bans that fall in the shard and writes, per row,
 * part[row] = {max, global index (u32 bits), sum exp(z - max), 0} (f32 x 4,
 * 16-byte aligned).  After an all-gather of the parts (rank-major:
 * parts[r][row]), madi_merge_shard_tail does the rest of madi_decode_tail: pos[row]
 * += 1, tokens[row][pos[row]] = the greedy token (the reference's tie order across
 * shards) and conf[row][pos[row]] = 1 / sum_r part_r.sum * exp(part_r.max - max)
 * (conf may be NULL).  Same tokens as madi_decode_tail over the gathered rows. */
int madi_shard_decode_tail(float *logits, int m, int n, uint32_t h0, int vocab, const uint32_t *tokens,
                           int64_t tok_stride, int max_len, const uint32_t *pos, uint32_t sample_begin,
                           uint32_t no_repeat_ngram, const uint32_t *suppress, int n_suppress, float *part,
                           void *stream);
int madi_merge_shard_tail(const float *parts, int world, int m, uint32_t *tokens, int64_t tok_stride, int max_len,
                          uint32_t *pos, float *conf, void *stream);

/* step_advance (graph_helpers.metal:60-62) for m <= 32 slots: pos[s] += 1. */
int madi_step_advance(uint32_t *pos, int m, void *stream);

/* ======================= rank-to-rank all-gather over NVLink ================= */
/* The column-split head's two exchanges per token step (hidden-state rows, per-row
 * parts) without a collective library.  No reference counterpart: the reference
 * runs one GPU; this replaces the all-gather the multi-GPU split head needs.
 * Every rank creates one object (ranks on DISTINCT GPUs of one node), hands its
 * 64-byte IPC handle to every peer (any host channel), and maps every peer's handle;
 * then every rank calls madi_xchg_allgather in the same order.  Each call stores this
 * rank's `bytes` of src into every rank's buffer over peer memory, raises a sequence
 * flag there, waits (bounded: MADI_EDEVICE at the next madi_sync on expiry) for every
 * peer's flag, and writes all ranks' rows, rank-major, to dst (world x bytes).  One
 * kernel per call, capturable in a CUDA graph.  bytes: a multiple of 16, <= cap. */
typedef struct madi_xchg madi_xchg;
int madi_xchg_create(int world, int rank, size_t cap_bytes, madi_xchg **out);
int madi_xchg_handle(const madi_xchg *x, void *handle64);
int madi_xchg_open(madi_xchg *x, int peer, const void *handle64);
int madi_xchg_allgather(madi_xchg *x, const void *src, size_t bytes, void *dst, void *stream);
/* Teardown in two steps: every rank unmaps its peers' buffers, the ranks meet (host
 * barrier), then every rank frees its own (destroy also unmaps what is still mapped). */
int madi_xchg_unmap(madi_xchg *x);
int madi_xchg_destroy(madi_xchg *x);

#ifdef __cplusplus
}
#endif
#endif /* MADI_Q8_H */
