"""CPU: the oracle against the reference's golden vectors and known answers.

Pins: tests/golden/quant_q8_golden.npz holds the outputs of the reference's own
quantiser (engine/metal/bench/quantize_q8.py, run by tests/golden/make_golden.py).
"""
import math
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quant_q8_golden.npz")


@pytest.mark.parametrize("case", ["normal", "wide", "edges"])
def test_quantiser_matches_reference_golden(oracle, case):
    g = np.load(GOLDEN)
    w = g[f"{case}_w_f16"].view(np.float16)
    qs, sc = oracle.quantize_q8(w)
    assert np.array_equal(qs, g[f"{case}_qs"]), "int8 quants differ from quantize_q8.py"
    assert np.array_equal(sc.view(np.uint16), g[f"{case}_scales_f16"]), "f16 scales differ from quantize_q8.py"


def test_quantiser_rounds_half_away_from_zero(oracle):
    # a block with max 127 has scale exactly 1.0: k+0.5 must round away from zero (Zig @round)
    w = np.zeros((1, 32), np.float16)
    w[0, 0] = 127.0
    w[0, 1:5] = [2.5, -2.5, 0.5, -0.5]
    qs, sc = oracle.quantize_q8(w)
    assert float(sc[0, 0]) == 1.0
    assert list(qs[0, 1:5]) == [3, -3, 1, -1]
    # an all-zero block keeps scale 1.0 (transcribe.zig:319)
    qs, sc = oracle.quantize_q8(np.zeros((2, 64), np.float16))
    assert (sc == 1.0).all() and (qs == 0).all()


def test_f16_conversions_exhaustive(oracle):
    L = oracle.lib()
    allh = np.arange(65536, dtype=np.uint16)
    ref = allh.view(np.float16).astype(np.float32)
    got = np.array([L.madi_orc_h2f(int(h)) for h in allh[::7]], np.float32)
    r = ref[::7]
    ok = np.isnan(r) | (got.view(np.uint32) == r.view(np.uint32))
    assert ok.all()
    x = np.random.default_rng(0).standard_normal(20000).astype(np.float32) * np.float32(2.0) ** \
        np.random.default_rng(1).integers(-30, 18, 20000).astype(np.float32)
    mine = np.array([L.madi_orc_f2h(float(v)) for v in x], np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(mine, x.astype(np.float16).view(np.uint16))


def test_gelu_matches_erf_definition(oracle):
    for v in np.linspace(-8, 8, 257):
        exact = 0.5 * v * (1 + math.erf(v / math.sqrt(2)))
        assert abs(oracle.gelu_erf(v) - exact) <= 2e-6 * max(1.0, abs(v))


def test_dequant_formula(oracle):
    rng = np.random.default_rng(3)
    qs = rng.integers(-127, 128, (40, 96), dtype=np.int8)
    sc = rng.uniform(1e-5, 3.0, (40, 3)).astype(np.float16)
    out = oracle.dequant_q8_f16(qs, sc)
    ref = (qs.astype(np.float32) * np.repeat(sc.astype(np.float32), 32, axis=1)).astype(np.float16).T
    assert np.array_equal(out.view(np.uint16), ref.view(np.uint16))


def test_linear_against_numpy(oracle):
    rng = np.random.default_rng(4)
    M, N, K = 37, 48, 96
    x = rng.standard_normal((M, K)).astype(np.float16)
    qs = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sc = rng.uniform(1e-4, 2e-3, (N, K // 32)).astype(np.float16)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float16)
    wdq = (qs.astype(np.float32) * np.repeat(sc.astype(np.float32), 32, axis=1)).astype(np.float16).astype(np.float64)
    acc = x.astype(np.float64) @ wdq.T
    y, yref = oracle.linear_f16(x, qs, sc, want_ref=True)
    np.testing.assert_allclose(y, acc, rtol=1e-12, atol=1e-12)
    assert np.abs(yref.astype(np.float64) - acc).max() <= 1e-3 * np.abs(acc).max()
    y = oracle.linear_f16(x, qs, sc, bias=b, epi=oracle.EPI_BIAS_RES, residual=r)
    np.testing.assert_allclose(y, acc + b + r.astype(np.float64), rtol=1e-12, atol=1e-12)
    y = oracle.linear_f16(x, qs, sc, bias=b, epi=oracle.EPI_BIAS_GELU)
    v = acc + b
    ge = 0.5 * v * (1 + np.vectorize(math.erf)(v / math.sqrt(2)))
    np.testing.assert_allclose(y, ge, atol=1e-6)


def test_gemv_against_numpy(oracle):
    rng = np.random.default_rng(5)
    M, N, K = 3, 40, 160
    x = rng.standard_normal((M, K)).astype(np.float32)
    qs = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sc = rng.uniform(1e-4, 2e-3, (N, K // 32)).astype(np.float16)
    w = qs.astype(np.float64) * np.repeat(sc.astype(np.float64), 32, axis=1)
    ref = x.astype(np.float64) @ w.T
    y, yf = oracle.gemv_q8(x, qs, sc, want_ref=True)
    np.testing.assert_allclose(y, ref, rtol=1e-12, atol=1e-12)
    assert np.abs(yf - ref).max() <= 1e-5 * np.abs(ref).max()       # Metal-order f32 restatement
    b = rng.standard_normal(N).astype(np.float32)
    r0 = rng.standard_normal((M, N)).astype(np.float32)
    y, yf = oracle.gemv_q8(x, qs, sc, bias=b, epi=oracle.EPI_BIAS_RES, res_in=r0, want_ref=True)
    np.testing.assert_allclose(y, ref + b + r0, rtol=1e-12, atol=1e-12)


def test_qkv_split(oracle):
    rng = np.random.default_rng(6)
    D = 64
    x = rng.standard_normal((2, D)).astype(np.float32)
    qs = rng.integers(-127, 128, (3 * D, D), dtype=np.int8)
    sc = rng.uniform(1e-4, 2e-3, (3 * D, D // 32)).astype(np.float16)
    qb = rng.standard_normal(D).astype(np.float32)
    vb = rng.standard_normal(D).astype(np.float32)
    pos = np.array([1, 4], np.uint32)
    q, kc, vc = oracle.gemv_q8_qkv(x, qs, sc, qb, vb, pos, 6)
    full = oracle.gemv_q8(x, qs, sc)
    np.testing.assert_allclose(q, full[:, :D] + qb, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(kc[4], full[1, D:2 * D], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(vc[1], full[0, 2 * D:] + vb, rtol=1e-12, atol=1e-12)
    assert np.isnan(kc[0]).all()


def _bitrev10(t):
    return int(format(t, "010b")[::-1], 2)


def _tree_argmax_py(l):
    """argmax_no_inc (graph_helpers.metal:64-95) as plain Python loops."""
    sv, si = [], []
    for t in range(1024):
        m, k = -np.inf, 0
        for i in range(t, len(l), 1024):
            if l[i] > m:
                m, k = l[i], i
        sv.append(m)
        si.append(k)
    s = 512
    while s:
        for t in range(s):
            if sv[t + s] > sv[t]:
                sv[t], si[t] = sv[t + s], si[t + s]
        s >>= 1
    return si[0]


def test_argmax_tree_tie_rule(oracle):
    """Ties resolve as the reference's 1024-lane tree does: the first index of
    the tied lane whose 10-bit id is smallest bit-reversed -- not the lowest index."""
    assert oracle.argmax(np.array([0.0, 3.0, 1.0, 3.0, -1.0], np.float32)) == 1
    assert oracle.argmax(np.array([0.0, 5.0, 5.0], np.float32)) == 2          # lane 2 (rev 256) beats lane 1 (rev 512)
    l = np.zeros(51866, np.float32)
    l[[5, 1029]] = 7.0                                                          # same lane: first index
    assert oracle.argmax(l) == 5
    rng = np.random.default_rng(11)
    for trial in range(6):
        l = rng.integers(-3, 4, 51866).astype(np.float32)                       # many ties at the max
        ties = np.flatnonzero(l == l.max())
        want = min(ties, key=lambda i: (_bitrev10(i % 1024), i))
        assert oracle.argmax(l) == want == _tree_argmax_py(l.tolist())
    assert oracle.argmax(np.full(51866, -np.inf, np.float32)) == 0


def test_argmax_conf_restatement(oracle):
    rng = np.random.default_rng(3)
    l = (rng.standard_normal(51866) * 4).astype(np.float32)
    tok, conf = oracle.argmax_conf(l)
    assert tok == int(np.argmax(l))
    p = 1.0 / np.exp(l.astype(np.float64) - l.max()).sum()
    assert abs(conf - p) <= 1e-5 * p


def test_emb_q8_restatement(oracle):
    rng = np.random.default_rng(4)
    qs = rng.integers(-127, 128, (10, 96), dtype=np.int8)
    sc = rng.uniform(1e-4, 2e-2, (10, 3)).astype(np.float16)
    out = oracle.emb_q8(qs, sc, 7)
    want = qs[7].astype(np.float64) * np.repeat(sc[7].astype(np.float64), 32)
    assert np.array_equal(out.astype(np.float64), want)      # exact: int8 x f16 fits f32


def test_logit_filter_restatement(oracle):
    NEG = np.float32(-3.4e38)
    V = 51866
    base = np.zeros(V, np.float32)

    def banned(out):
        return set(np.flatnonzero(out == NEG).tolist()) - set(range(50258, V))

    past = np.array([50258, 10, 20, 30, 40, 50, 60], np.uint32)
    out = oracle.logit_filter(base, past, 7, 1, 0)
    assert (out[50258:] == NEG).all() and banned(out) == set()
    assert banned(oracle.logit_filter(base, past, 4, 1, 0)) == {220, 50257}       # step < sample_begin + 4
    loop = np.array([50258, 7, 9, 9, 9], np.uint32)
    assert banned(oracle.logit_filter(base, loop, 5, 1, 0)) == {9}                 # anti-loop
    assert banned(oracle.logit_filter(base, loop, 5, 3, 0)) == {220, 50257}       # history before sample_begin
    ng = np.array([50258, 1, 2, 3, 1, 2, 3, 1], np.uint32)
    assert banned(oracle.logit_filter(base, ng, 8, 1, 2)) == {2}                   # bigram "1 2" seen -> ban 2
    assert banned(oracle.logit_filter(base, ng, 8, 1, 3)) == {2}                   # "3 1" was followed by 2
    ng3 = np.array([50258, 5, 6, 7, 5, 6], np.uint32)
    assert banned(oracle.logit_filter(base, ng3, 6, 1, 3)) == {7}                  # "5 6 7" then "5 6" -> ban 7
    assert banned(oracle.suppress(base, np.array([3, 99999, 11], np.uint32))) == {3, 11}   # out-of-range id skipped


def test_cpu_baseline_kernel_matches_exact(oracle):
    rng = np.random.default_rng(7)
    M, N, K = 64, 96, 256
    x = rng.standard_normal((M, K)).astype(np.float16)
    qs = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sc = rng.uniform(1e-4, 2e-3, (N, K // 32)).astype(np.float16)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    y = oracle.linear_f32_baseline(x, qs, sc, b, oracle.EPI_BIAS_GELU, nthreads=2)
    ex = oracle.linear_f16(x, qs, sc, b, oracle.EPI_BIAS_GELU)
    assert np.abs(y.astype(np.float64) - ex).max() <= 2e-3 * np.sqrt(np.mean(ex ** 2)) + np.abs(ex).max() * 2 ** -11


def test_oracle_bias_res_ln_restatement(oracle):
    """The residual + LayerNorm restatement (encoder_ops.metal:305-364): the f32
    residual update in the reference's order, and the LayerNorm against numpy."""
    g = np.random.default_rng(3)
    x = g.standard_normal((9, 384)).astype(np.float32)
    mo = g.standard_normal((9, 384)).astype(np.float16)
    b = (0.05 * g.standard_normal(384)).astype(np.float32)
    gamma = (1 + 0.1 * g.standard_normal(384)).astype(np.float32)
    beta = (0.1 * g.standard_normal(384)).astype(np.float32)
    x2, y = oracle.bias_res_ln(x, mo, b, gamma, beta, 1e-5)
    xe = (x + mo.astype(np.float32)) + b
    assert np.array_equal(x2, xe)
    m = xe.astype(np.float64).mean(1, keepdims=True)
    v = ((xe - m) ** 2).mean(1, keepdims=True)
    assert np.abs(y - ((xe - m) / np.sqrt(v + 1e-5) * gamma + beta)).max() < 1e-9
    x3, y3 = oracle.bias_res_ln(x, None, None, gamma, beta, 1e-5)
    assert np.array_equal(x3, x)
