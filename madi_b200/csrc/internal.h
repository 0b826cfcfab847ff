// internal.h -- launcher interfaces between the C-ABI layer (runtime.cu) and
// the kernel translation units.  Not part of the public ABI.
#pragma once
#include <cuda.h>
#include <mutex>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace madi {

// Whether launches use programmatic dependent launch (MADI_PDL=0 turns it off).
bool pdl_on();
// Streaming multiprocessors of the current device.
int num_sms();

// cudaLaunchKernelEx with the programmatic-serialization attribute (when on) and
// an optional cluster width along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster_x,
                     Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = pdl_on() ? 1 : 0;
    ++na;
    if (cluster_x > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = cluster_x;
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, fn, args...);
}

enum : int { kEpiNone = 0, kEpiBias = 1, kEpiBiasGelu = 2, kEpiBiasRes = 3 };
// Tensor-core path only: no epilogue, f32 output (logits of a vocab head with
// more than 8 token slots).
constexpr int kEpiNoneF32 = 4;
// Tensor-core path only: the encoder's f32 residual stream updated in place,
// y[m][n] = (r[m][n] + float(half(acc))) + bias[n] with r, y f32 (r may be y) --
// the residual add of bias_res_ln_f16 (encoder_ops.metal:343-347) on the f16
// projection output the reference's GEMM writes, moved into the GEMM's epilogue.
constexpr int kEpiResF32 = 5;

// ---------------------------------------------------------------- variant (b)
struct GemvArgs {
    const int8_t *qs;        // [N][K]
    const __half *scales;    // [N][K/32]
    const void *x;           // [M][K] f32 or f16
    void *y;                 // [M][N] f32 or f16 (QKV: q_out f32 [M][D])
    const void *residual;    // [M][N], y's type (EPI_BIAS_RES)
    const void *bias;        // [N] f32 or f16
    int N, K, M, ks;         // ks = thread-block cluster size along K (1, 2, 4, 8)
    int bias_f16;
    // QKV fusion (gemv_q8_qkv)
    const float *qb, *vb;
    float *kc, *vc;
    const uint32_t *pos;
    long long cache_stride;
    int D;
};
int gemv_pick_ks(int N, int K, int num_sms);
size_t gemv_smem_bytes(int M, int K, int cs, bool x_f32);
cudaError_t launch_gemv(const GemvArgs &a, bool x_f32, bool y_f32, int epi, bool qkv, cudaStream_t st, bool pdl);
// TMA-streamed tile kernel (q8_gemv_tile.cu): every shape with K % 256 == 0 whose
// x slice and one weight stage fit in shared memory, QKV included; same
// arithmetic and epilogues as launch_gemv.  Needs 16-byte aligned qs and scales.
bool gemv_tile_ok(int M, int N, int K, bool x_f32, int num_sms);
// x_r16: x f32, rounded to f16 when staged (the reference's batched decode rounds its
// activations to f16); then as f16 x.
cudaError_t launch_gemv_tile(const GemvArgs &a, bool x_f32, bool y_f32, int epi, bool qkv, int num_sms, int *dev_err,
                             cudaStream_t st, bool pdl, bool x_r16 = false);

// ---------------------------------------------------------------- variant (a)
struct GemmArgs {
    const __half *x;         // [M][K] f16
    const int8_t *qs;        // [N][K]
    const __half *scales;    // [N][K/32]
    const void *bias;        // [N] f32 or f16
    const void *residual;    // [M][N] f16 (f32 for kEpiResF32)
    __half *y;               // [M][N] f16 (f32 for kEpiNoneF32 / kEpiResF32)
    int M, N, K;
    int bias_f16;
    int *dev_err;            // device error word (bounded-wait expiry)
};
// Returns cudaErrorNotSupported if the tensor-map encoder is unavailable.
cudaError_t launch_gemm_tc(const GemmArgs &a, int epi, int num_sms, cudaStream_t st);
// The smallest M routed to variant (a) by madi_q8_linear.
constexpr int kGemmMinM = 9;
// The largest M the streaming skinny GEMM (q8_gemv_tile.cu) takes: two groups of 8
// token rows per weight fragment.
constexpr int kGemvMaxM = 16;

// ---------------------------------------------------------------- rank-to-rank all-gather (xchg.cu)
constexpr int kXchgMaxWorld = 8;
// Bytes of one rank's exchange buffer: 256-byte header (flags, call counter), then
// data[2][world][cap].
size_t xchg_buffer_bytes(int world, size_t cap);
// bases[r]: rank r's buffer as this rank maps it (bases[rank] its own).
cudaError_t launch_xchg_allgather(uint8_t *const *bases, int world, int rank, size_t cap, const void *src,
                                  size_t bytes, void *dst, int *dev_err, cudaStream_t st);

// ---------------------------------------------------------------- residual + LayerNorm (res_ln.cu)
constexpr int kLnMaxD = 2048;   // row width limit of the register-resident row kernel (D % 128 == 0)
// MO == nullptr: layer_norm_f16; else bias_res_ln_f16 (X updated in place).
cudaError_t launch_res_ln(float *X, const __half *MO, const float *bias, __half *Y, const float *gamma,
                          const float *beta, int rows, int D, float eps, cudaStream_t st);
cudaError_t launch_res_ln_f32(float *X, const float *MO, const float *bias, float *Y, const float *gamma,
                              const float *beta, int rows, int D, float eps, cudaStream_t st);
// MO f32, Y f16 (round to nearest): the decoder's forms feeding f16-activation projections.
cudaError_t launch_res_ln_f32_y16(float *X, const float *MO, const float *bias, __half *Y, const float *gamma,
                                  const float *beta, int rows, int D, float eps, cudaStream_t st);

// ---------------------------------------------------------------- decode-step primitives (decode_step.cu)
constexpr int kWhisperVocab = 51866;   // VOCAB of graph_helpers.metal:9 (the by-name kernels assume it)
// tok_len: entries readable per slot row of `tokens`; rows: embedding rows.
cudaError_t launch_emb_q8(float *out, const int8_t *qs, const __half *scales, const uint32_t *tokens,
                          const uint32_t *pos, int dim, int rows, int m, long long tok_stride, long long tok_len,
                          const float *pos_emb, int max_pos, cudaStream_t st);
cudaError_t launch_emb_f16(float *out, const __half *emb, const uint32_t *tokens, const uint32_t *pos, int dim,
                           int rows, long long tok_len, cudaStream_t st);
cudaError_t launch_pos_add(float *out, const float *pos_emb, const uint32_t *pos, int dim, int max_pos, cudaStream_t st);
cudaError_t launch_step_advance(uint32_t *pos, int m, cudaStream_t st);
cudaError_t launch_argmax(const float *logits, uint32_t *tokens, float *conf, const uint32_t *pos, int V, int max_len,
                          int m, long long stride, cudaStream_t st);
cudaError_t launch_suppress(float *logits, const uint32_t *ids, int n, int V, int rows, cudaStream_t st);
cudaError_t launch_logit_filter(float *logits, const uint32_t *past, const uint32_t *step_ptr, uint32_t sample_begin,
                                uint32_t no_repeat_ngram, int V, int past_len, int rows, long long past_stride,
                                cudaStream_t st);
// ---- decoder attention (attn.cu); head_dim 64
constexpr int kAttnMaxChunk = 256;   // keys per CTA of a cross-attention cluster (seqlen <= 8 * 256)
constexpr int kAttnMaxTok = 512;     // self-attention keys per slot
int attn_cluster_size(int seqlen);   // CTAs per (slot, head); 0 if seqlen is too long
cudaError_t launch_cross_attn(float *out, const float *q, const void *kc, const void *vc, bool kv_f16, float *scores,
                              int slots, int seqlen, int kvd, int nkv, int nh, int *dev_err, cudaStream_t st);
cudaError_t launch_cross_attn_part(float *part, const float *q, const void *kc, const void *vc, bool kv_f16,
                                   float *sc_raw, int write_sc, int seqlen, int kvd, int nkv, int nh, int nsplit,
                                   cudaStream_t st);
cudaError_t launch_cross_attn_reduce(float *out, const float *part, int nsplit, float *sc, int seqlen, int write_sc,
                                     int nh, cudaStream_t st);
// Split form with the partials in a fixed device array (attn.cu): heads x nsplit at
// most kSplitStaticMax.  Looks the array's device address up on each device's
// first call (again when the device's context changed); cudaErrorInvalidDevice
// unless the current device is `device` (the one the library is bound to).
constexpr int kSplitStaticMax = 2048;
cudaError_t launch_cross_attn_split_static(float *out, const float *q, const void *kc, const void *vc, float *sc,
                                           int seqlen, int kvd, int nkv, int nh, int nsplit, int device,
                                           cudaStream_t st);
// Drops the looked-up addresses (madi_cleanup).
void forget_split_static_addresses();
cudaError_t launch_self_attn(float *out, const float *q, const void *kc, const void *vc, bool kv_f16,
                             const uint32_t *pos, int slots, int kvd, int nkv, int nh, int max_tok, int *dev_err,
                             cudaStream_t st);
// ---- encoder self-attention on the tensor cores (flash_enc.cu); head_dim 64
cudaError_t launch_flash_enc(const __half *q, const __half *k, const __half *v, int stride, __half *out,
                             int out_stride, int seq, int heads, int chunks, int *dev_err, cudaStream_t st);
// step_advance + logit_filter_indirect + suppress_list + argmax_conf for m slots in
// one launch (V <= decode_tail_max_vocab()).
int decode_tail_max_vocab();
cudaError_t launch_decode_tail(float *logits, int m, int V, uint32_t *tokens, long long stride, int max_len,
                               uint32_t *pos, float *conf, uint32_t sample_begin, uint32_t no_repeat_ngram,
                               const uint32_t *sup, int nsup, cudaStream_t st);
// The same tail over one column shard [h0, h0 + n) of a V-token vocabulary: per row
// the shard's (max, global index, exp sum against its max) into part[row]; then
// the merge of the world shards' parts (rank-major) with step_advance and the
// token / confidence writes.
cudaError_t launch_shard_tail(float *logits, int m, int n, uint32_t h0, int V, const uint32_t *tokens,
                              long long stride, int max_len, const uint32_t *pos, uint32_t sample_begin,
                              uint32_t no_repeat_ngram, const uint32_t *sup, int nsup, float4 *part, cudaStream_t st);
cudaError_t launch_merge_tail(const float4 *part, int world, int m, uint32_t *tokens, long long stride, int max_len,
                              uint32_t *pos, float *conf, cudaStream_t st);
cudaError_t launch_shard_argmax(const float *logits, long long row_stride, int n, uint32_t h0, int m, float *vals,
                                uint32_t *idx, cudaStream_t st);
cudaError_t launch_merge_argmax(const float *vals, const uint32_t *idx, int world, int m, uint32_t *tokens,
                                cudaStream_t st);

// ---------------------------------------------------------------- misc kernels
cudaError_t launch_dequant_f16(const int8_t *qs, const __half *scales, int N, int K, __half *out, cudaStream_t st);
cudaError_t launch_quantize_f16(const __half *w, int rows, int dim, int8_t *qs, __half *scales, cudaStream_t st);

// One-time set-up shared by every host thread: `init` runs once per call site (per
// template instantiation inside a template) and its status is returned to every
// later caller; concurrent first calls wait for the one that runs it.  The library
// binds one device per process (madi_init), so set-up that belongs to a device
// (function attributes, occupancy queries) is done for that device.
template <typename F>
inline cudaError_t run_once(std::once_flag &flag, cudaError_t &status, F &&init) {
    std::call_once(flag, [&] { status = init(); });
    return status;
}

// Driver entry point for cuTensorMapEncodeTiled (resolved lazily through the
// runtime, so the library needs no link-time libcuda).
typedef CUresult (*PFN_encodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
PFN_encodeTiled tensor_map_encoder();

}  // namespace madi
