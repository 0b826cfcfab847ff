"""numpy front-end for the C oracle (oracle/q8_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU legs may import this module;
madi_b200 never does.  See q8_oracle.c's header for what each function
restates (reference file:line) and for the parity status (quantiser pinned to
the reference's quantize_q8.py outputs; linear / GEMV arithmetic unpinned
restatements, because the reference's Metal kernels cannot run here).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libmadi_oracle.so")

EPI_NONE, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RES = 0, 1, 2, 3

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.madi_orc_h2f.argtypes, L.madi_orc_h2f.restype = [ctypes.c_uint16], F
        L.madi_orc_f2h.argtypes, L.madi_orc_f2h.restype = [F], ctypes.c_uint16
        L.madi_orc_quantize_q8.argtypes = [P, I, I, P, P]
        L.madi_orc_dequant_q8_f16.argtypes = [P, P, I, I, P]
        L.madi_orc_gelu_erf.argtypes, L.madi_orc_gelu_erf.restype = [F], F
        L.madi_orc_linear_f16.argtypes = [P, I, I, P, P, I, P, I, P, P, P]
        L.madi_orc_gemv_q8.argtypes = [P, I, P, P, I, I, P, I, P, P, P]
        L.madi_orc_gemv_q8_qkv.argtypes = [P, I, P, P, I, P, P, P, P, P, P]
        L.madi_orc_argmax.argtypes, L.madi_orc_argmax.restype = [P, I], I
        L.madi_orc_argmax_conf.argtypes, L.madi_orc_argmax_conf.restype = [P, I, P], I
        L.madi_orc_emb_q8.argtypes = [P, P, I, ctypes.c_uint32, P]
        L.madi_orc_suppress.argtypes = [P, I, P, I]
        L.madi_orc_logit_filter.argtypes = [P, I, P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
        L.madi_orc_linear_f32_baseline.argtypes = [P, I, I, P, P, I, P, I, P, P, I]
        L.madi_orc_bias_res_ln.argtypes = [P, P, P, P, P, I, I, F, P]
        L.madi_orc_linear_f32_baseline.restype = I
        L.madi_orc_max_threads.restype = I
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


def quantize_q8(w_f16: np.ndarray):
    """transcribe.zig:309-327 quantInto.  w f16 [rows][dim] -> (qs int8, scales f16)."""
    w = _c(w_f16, np.float16)
    rows, dim = w.shape
    assert dim % 32 == 0
    qs = np.empty((rows, dim), np.int8)
    sc = np.empty((rows, dim // 32), np.uint16)
    lib().madi_orc_quantize_q8(_p(w.view(np.uint16)), rows, dim, _p(qs), _p(sc))
    return qs, sc.view(np.float16)


def dequant_q8_f16(qs, scales):
    """q8_gemm.metal:12-27: -> f16 [K][N] (transposed)."""
    qs = _c(qs, np.int8)
    sc = _c(scales, np.float16)
    N, K = qs.shape
    out = np.empty((K, N), np.uint16)
    lib().madi_orc_dequant_q8_f16(_p(qs), _p(sc.view(np.uint16)), N, K, _p(out))
    return out.view(np.float16)


def gelu_erf(x: float) -> float:
    return lib().madi_orc_gelu_erf(float(x))


def linear_f16(X, qs, scales, bias=None, epi=EPI_NONE, residual=None, want_ref=False):
    """Encoder linear.  Returns y_exact f64 [M][N] (and y_ref f16 if want_ref)."""
    X = _c(X, np.float16)
    qs = _c(qs, np.int8)
    sc = _c(scales, np.float16)
    M, K = X.shape
    N = qs.shape[0]
    b = _c(bias, np.float32)
    r = _c(residual, np.float16)
    y = np.empty((M, N), np.float64)
    yr = np.empty((M, N), np.uint16) if want_ref else None
    lib().madi_orc_linear_f16(_p(X.view(np.uint16)), M, K, _p(qs), _p(sc.view(np.uint16)), N, _p(b), epi,
                              None if r is None else _p(r.view(np.uint16)), _p(y), _p(yr))
    return (y, yr.view(np.float16)) if want_ref else y


def gemv_q8(x, qs, scales, bias=None, epi=EPI_NONE, res_in=None, want_ref=False):
    """Decode GEMV family in f32 semantics.  x f32 [M][K] -> f64 [M][N] (+ f32 ref)."""
    x = _c(np.atleast_2d(x), np.float32)
    qs = _c(qs, np.int8)
    sc = _c(scales, np.float16)
    M, K = x.shape
    N = qs.shape[0]
    b = _c(bias, np.float32)
    r = _c(res_in, np.float32)
    y = np.empty((M, N), np.float64)
    yr = np.empty((M, N), np.float32) if want_ref else None
    lib().madi_orc_gemv_q8(_p(x), M, _p(qs), _p(sc.view(np.uint16)), N, K, _p(b), epi, _p(r), _p(y), _p(yr))
    return (y, yr) if want_ref else y


def gemv_q8_qkv(x, qs, scales, qb, vb, pos, cache_rows):
    """graph_helpers.metal:527-567.  Returns (q f64 [M][D], kc f64 [rows][D], vc f64 [rows][D]);
    cache rows not written stay NaN."""
    x = _c(np.atleast_2d(x), np.float32)
    qs = _c(qs, np.int8)
    sc = _c(scales, np.float16)
    M, D = x.shape
    pos = _c(pos, np.uint32)
    q = np.empty((M, D), np.float64)
    kc = np.full((cache_rows, D), np.nan)
    vc = np.full((cache_rows, D), np.nan)
    lib().madi_orc_gemv_q8_qkv(_p(x), M, _p(qs), _p(sc.view(np.uint16)), D, _p(_c(qb, np.float32)),
                               _p(_c(vb, np.float32)), _p(pos), _p(q), _p(kc), _p(vc))
    return q, kc, vc


def argmax(logits) -> int:
    """Greedy token with the reference's 1024-lane tree tie rule (argmax_no_inc)."""
    l = _c(logits, np.float32)
    return lib().madi_orc_argmax(_p(l), l.size)


def argmax_conf(logits):
    """(token, confidence) as argmax_conf computes them (graph_helpers.metal:785-821)."""
    l = _c(logits, np.float32)
    c = ctypes.c_float()
    tok = lib().madi_orc_argmax_conf(_p(l), l.size, ctypes.byref(c))
    return tok, c.value


def emb_q8(qs, scales, tok: int):
    """One dequantised Q8 embedding row as f32 (emb_lookup_indirect_q8)."""
    qs = _c(qs, np.int8)
    sc = _c(scales, np.float16)
    out = np.empty(qs.shape[1], np.float32)
    lib().madi_orc_emb_q8(_p(qs), _p(sc.view(np.uint16)), qs.shape[1], int(tok), _p(out))
    return out


def suppress(logits, ids):
    """suppress_list on a copy of one logits row."""
    l = _c(logits, np.float32).copy()
    i = _c(ids, np.uint32)
    lib().madi_orc_suppress(_p(l), l.size, _p(i), i.size)
    return l


def logit_filter(logits, past, step: int, sample_begin: int, no_repeat_ngram: int = 0):
    """logit_filter_indirect on a copy of one logits row (graph_helpers.metal:109-160)."""
    l = _c(logits, np.float32).copy()
    p = _c(past, np.uint32)
    if step > p.size:
        raise ValueError("step beyond the token history")
    lib().madi_orc_logit_filter(_p(l), l.size, _p(p), int(step), int(sample_begin), int(no_repeat_ngram))
    return l


def linear_f32_baseline(X, qs, scales, bias=None, epi=EPI_NONE, residual=None, nthreads=None):
    """The reference's CPU loop (f32 dequant + accumulate) -- the timed CPU baseline."""
    X = _c(X, np.float16)
    qs = _c(qs, np.int8)
    sc = _c(scales, np.float16)
    M, K = X.shape
    N = qs.shape[0]
    y = np.empty((M, N), np.uint16)
    nt = nthreads or lib().madi_orc_max_threads()
    r = _c(residual, np.float16)
    lib().madi_orc_linear_f32_baseline(_p(X.view(np.uint16)), M, K, _p(qs), _p(sc.view(np.uint16)), N,
                                       _p(_c(bias, np.float32)), epi,
                                       None if r is None else _p(r.view(np.uint16)), _p(y), nt)
    return y.view(np.float16)


def max_threads() -> int:
    return lib().madi_orc_max_threads()


def bias_res_ln(x, mo=None, bias=None, gamma=None, beta=None, eps=1e-5):
    """bias_res_ln_f16 / layer_norm_f16 restated (encoder_ops.metal:305-364).
    x f32 [rows][d] (not modified here); mo f16 [rows][d] or None.  Returns
    (x updated in f32, y exact in f64)."""
    x2 = _c(x, np.float32).copy()
    rows, d = x2.shape
    y = np.empty((rows, d), dtype=np.float64)
    mo_c = None if mo is None else _c(mo, np.float16).view(np.uint16)
    lib().madi_orc_bias_res_ln(_p(x2), None if mo_c is None else _p(mo_c),
                               None if bias is None else _p(_c(bias, np.float32)),
                               _p(_c(gamma, np.float32)), _p(_c(beta, np.float32)), rows, d, float(eps), _p(y))
    return x2, y


def bias_res_ln_f32(x, mo=None, bias=None, gamma=None, beta=None, eps=1e-5):
    """bias_res_ln / layer_norm, the decoder's f32 forms (encoder_ops.metal:14-120):
    x + mo + bias in the reference's f32 order ((x + mo) + bias), then the LayerNorm
    in f64.  Returns (x updated in f32, y exact in f64)."""
    x2 = np.array(x, dtype=np.float32, copy=True)
    if mo is not None:
        x2 = (x2 + np.asarray(mo, np.float32)) + np.asarray(bias, np.float32)
    xd = x2.astype(np.float64)
    mean = xd.mean(axis=1, keepdims=True)
    var = ((xd - mean) ** 2).mean(axis=1, keepdims=True)
    y = (xd - mean) / np.sqrt(var + float(np.float32(eps))) * np.asarray(gamma, np.float64) + np.asarray(beta,
                                                                                                      np.float64)
    return x2, y


def _head_kv(kc, vc, h, nh, nkv, hdd):
    kvh = h * nkv // nh
    return kc[..., kvh * hdd:(kvh + 1) * hdd], vc[..., kvh * hdd:(kvh + 1) * hdd]


def cross_attn(q, kc, vc, nh, nkv=None, hdd=64):
    """flash_cross_attn / _f16kv / _f16kv_batched (decoder_ops.metal:194-325, 459-531)
    restated in f64: per slot and head, s_t = q_h . k_t * rsqrt(hdd), p = softmax(s)
    (the reference's exp2((s - max) * log2 e) / sum), out_h = sum_t p_t v_t.
    q [slots][nh*hdd]; kc, vc [slots][seqlen][kvd].  Returns (out [slots][nh*hdd],
    scores [slots][nh][seqlen])."""
    nkv = nkv or nh
    q = np.asarray(q, np.float64)
    kc = np.asarray(kc, np.float64)
    vc = np.asarray(vc, np.float64)
    slots, seqlen, _ = kc.shape
    out = np.empty((slots, nh * hdd))
    sc = np.empty((slots, nh, seqlen))
    for h in range(nh):
        K, V = _head_kv(kc, vc, h, nh, nkv, hdd)
        s = np.einsum("bd,btd->bt", q[:, h * hdd:(h + 1) * hdd], K) / np.sqrt(hdd)
        e = np.exp(s - s.max(axis=1, keepdims=True))
        p = e / e.sum(axis=1, keepdims=True)
        sc[:, h] = p
        out[:, h * hdd:(h + 1) * hdd] = np.einsum("bt,btd->bd", p, V)
    return out, sc


def self_attn(q, kc, vc, pos, nh, nkv=None, hdd=64):
    """gpu_attention (decoder_ops.metal:81-149) restated in f64: slot b attends its
    cache rows 0..pos[b] (at most the cache length).  kc, vc [slots][max_tok][kvd]."""
    nkv = nkv or nh
    kc = np.asarray(kc, np.float64)
    vc = np.asarray(vc, np.float64)
    out = np.empty((kc.shape[0], nh * hdd))
    for b, p in enumerate(np.asarray(pos).tolist()):
        n = min(int(p) + 1, kc.shape[1])
        o, _ = cross_attn(np.asarray(q, np.float64)[b:b + 1], kc[b:b + 1, :n], vc[b:b + 1, :n], nh, nkv, hdd)
        out[b] = o[0]
    return out


def flash_attn_enc(q, k, v, heads, seq, hdd=64):
    """m4_flash_enc (m4_gemm.metal:255-407) restated without tiling in f64: per chunk
    and head, softmax(Q K^T * 0.125) V.  The unrounded result (the reference's
    kernel rounds P to f16 inside its online softmax; the parity gate is measured
    against this exact value).  q / k / v [chunks * seq][heads * hdd]."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    out = np.empty((q.shape[0], heads * hdd))
    for c in range(q.shape[0] // seq):
        r = slice(c * seq, (c + 1) * seq)
        for h in range(heads):
            cs = slice(h * hdd, (h + 1) * hdd)
            s = (q[r, cs] @ k[r, cs].T) * 0.125
            e = np.exp(s - s.max(axis=1, keepdims=True))
            out[r, cs] = (e @ v[r, cs]) / e.sum(axis=1, keepdims=True)
    return out

