"""Variant (b) parity: decode GEMV / skinny GEMM (M <= 16) against the oracle.

The oracle restates graph_helpers.metal's f32 GEMV family; the gate
(tests/gate.py) is max |y - y_exact| <= 2e-3 * RMS(y_exact) with y_exact the
f64 result (beyond the final rounding for f16 outputs).  The
kernel keeps f32 semantics (exact int8 weights, f32 block scales, split-f16
activations), so in practice it lands near 1e-6 * RMS; a tighter diagnostic
bound of 5e-5 is asserted too, to catch precision regressions early.
"""
import numpy as np
import pytest

from madi_b200 import synth

from tests.gate import check as gate_check

TIGHT = 5e-5
pytestmark = pytest.mark.gpu


def _t(a, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _check(y_gpu, y_exact, what, tight=True, f16_out=False):
    ex, raw = gate_check(y_gpu.float().cpu().numpy(), y_exact, what, f16_out=f16_out)
    if tight:
        assert raw <= TIGHT, f"{what}: max|err|/RMS {raw:.2e} above the f32-semantics bound {TIGHT}"
    return raw


def _case(madi, oracle, M, N, K, epi, x_dt=np.float32, y_dt=np.float32, seed=0):
    import torch
    from madi_b200 import q8
    qs, sc = synth.q8_weight(N, K, seed + 11)
    x = synth.activations(M, K, seed + 12, dtype=x_dt)
    b = synth.bias(N, seed + 13)
    res = synth.activations(M, N, seed + 14, dtype=y_dt) if epi == q8.EPI_BIAS_RES else None
    W = q8.Q8Weight(_t(qs), _t(sc))
    out = torch.empty((M, N), dtype=torch.float32 if y_dt == np.float32 else torch.float16, device="cuda")
    if res is not None:
        out.copy_(_t(res))
    q8.linear(W, _t(x), bias=_t(b) if epi else None, epi=epi,
              residual=out if res is not None else None, out=out)
    torch.cuda.synchronize()
    y_exact = oracle.gemv_q8(x.astype(np.float32), qs, sc, bias=b, epi=epi,
                             res_in=None if res is None else res.astype(np.float32))
    # f16 inputs/outputs round: only the standard gate applies
    tight = x_dt == np.float32 and y_dt == np.float32
    return _check(out, y_exact, f"M={M} N={N} K={K} epi={epi}", tight=tight, f16_out=y_dt == np.float16)


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 7, 8])
@pytest.mark.parametrize("name,N,K", synth.decoder_shapes())
def test_decoder_shapes(madi, oracle, M, name, N, K):
    epi = {"qkv": 0, "o": 0, "cq": 1, "co": 0, "fc1": 2, "fc2": 3}[name]
    _case(madi, oracle, M, N, K, epi, seed=M * 7 + N)


@pytest.mark.parametrize("M", [1, 8])
def test_vocab_head(madi, oracle, M):
    _case(madi, oracle, M, synth.VOCAB, synth.D_MODEL, 0, seed=M)


@pytest.mark.parametrize("x_dt,y_dt", [(np.float16, np.float32), (np.float32, np.float16), (np.float16, np.float16)])
def test_dtypes(madi, oracle, x_dt, y_dt):
    for epi in (0, 1, 2, 3):
        _case(madi, oracle, 4, 1280, 1280, epi, x_dt=x_dt, y_dt=y_dt, seed=epi)


@pytest.mark.parametrize("N,K", [(1, 32), (17, 64), (100, 96), (1000, 2080), (51866, 32)])
def test_ragged_shapes(madi, oracle, N, K):
    _case(madi, oracle, 3, N, K, 1, seed=N + K)


def _args_gemv(mtl, out, Q, S, X, N, K, bias=None):
    a = [mtl.Arg.buf(out), mtl.Arg.buf(Q), mtl.Arg.buf(S), mtl.Arg.buf(X)]
    if bias is not None:
        a.append(mtl.Arg.buf(bias))
    return a + [mtl.Arg.u32(N), mtl.Arg.u32(K)]


def test_reference_gemv_family_through_dispatch(madi, oracle):
    """gemv_q8 / _bias / _bias_gelu / _bias_res / logit_gemv_q8 by name, with the
    reference's argument orders and grids (decoder.zig:155-200)."""
    import torch
    from madi_b200 import backend as mtl
    N, K = 5120, 1280
    qs, sc = synth.q8_weight(N, K, 21)
    x = synth.activations(1, K, 22, np.float32)[0]
    b = synth.bias(N, 23)
    Q, S, X, B = _t(qs), _t(sc), _t(x), _t(b)
    out = torch.zeros(N, dtype=torch.float32, device="cuda")
    grid, block = ((N + 7) // 8, 1, 1), (256, 1, 1)
    for name, epi in (("gemv_q8", 0), ("gemv_q8_bias", 1), ("gemv_q8_bias_gelu", 2)):
        out.zero_()
        mtl.dispatch(mtl.get_function(name), grid, block, _args_gemv(mtl, out, Q, S, X, N, K, B if epi else None))
        mtl.sync(10000)
        _check(out, oracle.gemv_q8(x, qs, sc, bias=b, epi=epi)[0], name)
    r0 = synth.activations(1, N, 24, np.float32)[0]
    out.copy_(_t(r0))
    mtl.dispatch(mtl.get_function("gemv_q8_bias_res"), grid, block, _args_gemv(mtl, out, Q, S, X, N, K, B))
    mtl.sync(10000)
    _check(out, oracle.gemv_q8(x, qs, sc, bias=b, epi=3, res_in=r0)[0], "gemv_q8_bias_res")
    # vocab head
    V, Dm = synth.VOCAB, synth.D_MODEL
    hq, hs = synth.q8_weight(V, Dm, 25)
    hx = synth.activations(1, Dm, 26, np.float32)[0]
    logits = torch.empty(V, dtype=torch.float32, device="cuda")
    mtl.dispatch(mtl.get_function("logit_gemv_q8"), ((V + 7) // 8, 1, 1), block,
                 [mtl.Arg.buf(logits), mtl.Arg.buf(_t(hq)), mtl.Arg.buf(_t(hs)), mtl.Arg.buf(_t(hx)),
                  mtl.Arg.u32(V), mtl.Arg.u32(Dm)])
    mtl.sync(10000)
    ex = oracle.gemv_q8(hx, hq, hs)[0]
    _check(logits, ex, "logit_gemv_q8")
    assert int(torch.argmax(logits).item()) == oracle.argmax(ex.astype(np.float32))


@pytest.mark.parametrize("M", [9, 12, 16])
@pytest.mark.parametrize("name,N,K", synth.decoder_shapes())
def test_decoder_shapes_two_token_groups(madi, oracle, M, name, N, K):
    """9..16 token rows: each weight fragment feeds two MMAs (tokens 0..7, 8..15),
    with the second group partly empty below 16."""
    epi = {"qkv": 0, "o": 0, "cq": 1, "co": 0, "fc1": 2, "fc2": 3}[name]
    _case(madi, oracle, M, N, K, epi, seed=M * 5 + N)


@pytest.mark.parametrize("M,N,K,epi,x_dt,y_dt", [
    (16, 51866, 1280, 0, np.float32, np.float32),   # vocab head, persistent ring
    (13, 40010, 1536, 3, np.float16, np.float16),   # ragged last tile, f16 in / out
    (10, 300, 1024, 1, np.float32, np.float32),     # 4-CTA clusters split K
    (16, 1280, 5120, 3, np.float32, np.float32),    # fc2 shape, f32 x
    (11, 37, 2048, 2, np.float16, np.float32),
    (15, 1280, 5120, 3, np.float16, np.float32),    # fc2, f16 activations: 4-CTA clusters, two units each
    (12, 1270, 5120, 0, np.float16, np.float16),    # the same plan, last tile ragged
    (16, 1264, 4096, 1, np.float16, np.float32),    # 79 tiles: the last cluster has one unit
])
def test_two_token_group_plans(madi, oracle, M, N, K, epi, x_dt, y_dt):
    _case(madi, oracle, M, N, K, epi, x_dt=x_dt, y_dt=y_dt, seed=N + K + 3 * M)


@pytest.mark.parametrize("M", [1, 3, 8, 12, 16])
@pytest.mark.parametrize("name,N,K", synth.decoder_shapes() + [("head", 51866, 1280)])
def test_f32_rounded_to_f16_on_load(madi, oracle, M, name, N, K):
    """MADI_F32_AS_F16: f32 x rounded to f16 as it is staged (the batched decode's f16
    activations), then the f16 path; against the oracle on the f16-rounded x."""
    import torch
    from madi_b200 import q8
    epi = {"qkv": 0, "o": 0, "cq": 1, "co": 0, "fc1": 2, "fc2": 3, "head": 0}[name]
    qs, sc = synth.q8_weight(N, K, M + N + 5)
    x = synth.activations(M, K, M + N + 6, dtype=np.float32) * 3.0
    b = synth.bias(N, M + N + 7)
    res = synth.activations(M, N, M + N + 8, dtype=np.float32) if epi == q8.EPI_BIAS_RES else None
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    if res is not None:
        out.copy_(_t(res))
    q8.linear(q8.Q8Weight(_t(qs), _t(sc)), _t(x), bias=_t(b) if epi else None, epi=epi,
              residual=out if res is not None else None, out=out, x_round16=True)
    torch.cuda.synchronize()
    x16 = x.astype(np.float16).astype(np.float32)
    y_exact = oracle.gemv_q8(x16, qs, sc, bias=b, epi=epi, res_in=res)
    _check(out, y_exact, f"round16 M={M} {name}")


def test_qkv_kv_store(madi, oracle):
    """gemv_q8_qkv: q+qb -> q_out, k -> kc[pos], v+vb -> vc[pos] (pos read on device)."""
    import torch
    from madi_b200 import backend as mtl, q8
    D, T = 1280, 448
    qs, sc = synth.q8_weight(3 * D, D, 31)
    qb, vb = synth.bias(D, 32), synth.bias(D, 33)
    # single slot through the reference name
    x = synth.activations(1, D, 34, np.float32)
    kc = torch.full((T, D), float("nan"), device="cuda")
    vc = torch.full((T, D), float("nan"), device="cuda")
    pos = torch.tensor([17], dtype=torch.int32, device="cuda")
    q_out = torch.empty(D, device="cuda")
    mtl.dispatch(mtl.get_function("gemv_q8_qkv"), ((3 * D + 7) // 8, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(q_out), mtl.Arg.buf(_t(qs)), mtl.Arg.buf(_t(sc)), mtl.Arg.buf(_t(x)),
                  mtl.Arg.buf(_t(qb)), mtl.Arg.buf(_t(vb)), mtl.Arg.buf(kc), mtl.Arg.buf(vc),
                  mtl.Arg.buf(pos), mtl.Arg.u32(D)])
    mtl.sync(10000)
    q_ex, k_ex, v_ex = oracle.gemv_q8_qkv(x, qs, sc, qb, vb, np.array([17], np.uint32), T)
    _check(q_out, q_ex[0], "q")
    _check(kc[17], k_ex[17], "k cache row")
    _check(vc[17], v_ex[17], "v cache row")
    assert torch.isnan(kc[16]).all() and torch.isnan(vc[18]).all(), "other cache rows must be untouched"
    # batched slots: per-slot caches and positions (5 slots, then 12: two token groups)
    for M, posb in [(5, np.array([0, 3, 447, 10, 200], np.uint32)),
                    (12, np.array([0, 3, 447, 10, 200, 1, 2, 5, 8, 13, 21, 34], np.uint32))]:
        _qkv_slots(oracle, qs, sc, qb, vb, D, T, M, posb)
    # the batched decode's f16-rounded activations
    _qkv_slots(oracle, qs, sc, qb, vb, D, T, 12, np.arange(12, dtype=np.uint32) * 7, round16=True)


def _qkv_slots(oracle, qs, sc, qb, vb, D, T, M, posb, round16=False):
    import torch
    from madi_b200 import q8
    xb = synth.activations(M, D, 35 + M, np.float32)
    kcb = torch.full((M, T, D), float("nan"), device="cuda")
    vcb = torch.full((M, T, D), float("nan"), device="cuda")
    W = q8.Q8Weight(_t(qs), _t(sc))
    qo = q8.qkv(W, _t(xb), _t(qb), _t(vb), kcb, vcb, _t(posb.astype(np.int32)), x_round16=round16)
    if round16:
        xb = xb.astype(np.float16).astype(np.float32)
    torch.cuda.synchronize()
    for s in range(M):
        q_ex, k_ex, v_ex = oracle.gemv_q8_qkv(xb[s:s + 1], qs, sc, qb, vb, posb[s:s + 1], T)
        _check(qo[s], q_ex[0], f"slot {s} q")
        _check(kcb[s, posb[s]], k_ex[posb[s]], f"slot {s} k")
        _check(vcb[s, posb[s]], v_ex[posb[s]], f"slot {s} v")


@pytest.mark.parametrize("M,epi,x_dt,y_dt", [(8, 1, np.float32, np.float32), (3, 2, np.float32, np.float32),
                                             (8, 3, np.float32, np.float32), (5, 0, np.float16, np.float32),
                                             (2, 1, np.float32, np.float16), (1, 3, np.float16, np.float16)])
def test_large_n_streaming_path(madi, oracle, M, epi, x_dt, y_dt):
    """Many more 16-row tiles than CTA slots: the TMA tile kernel runs persistent
    (two CTAs per SM, a ring of stages each); N = 40010 leaves a ragged last tile
    (10 rows) that the TMA unit zero-fills."""
    _case(madi, oracle, M, 40010, 1536, epi, x_dt=x_dt, y_dt=y_dt, seed=M * 13 + epi)


@pytest.mark.parametrize("M,N,K,epi,x_dt,y_dt", [
    (3, 300, 1024, 1, np.float32, np.float32),     # 19 tiles: 4-CTA clusters split K (256 each)
    (5, 37, 2048, 2, np.float32, np.float32),      # 3 tiles, the last ragged, 4-way split
    (2, 1280, 5120, 3, np.float32, np.float32),    # fc2 shape, 2-way split
    (8, 1280, 5120, 3, np.float16, np.float32),    # fc2 with f16 activations, 2-way split
    (7, 1280, 5120, 0, np.float16, np.float16),
    (4, 4000, 4096, 1, np.float32, np.float32),    # persistent, one CTA per SM (x slice too big for two)
    (1, 2048, 256, 0, np.float32, np.float32),     # K = 256: one box, one block per warp
])
def test_tile_kernel_plans(madi, oracle, M, N, K, epi, x_dt, y_dt):
    """The tile kernel's launch plans: thread-block clusters splitting K (partial
    sums pushed into rank 0), one unit per CTA, persistent rings."""
    _case(madi, oracle, M, N, K, epi, x_dt=x_dt, y_dt=y_dt, seed=N + K + M)
