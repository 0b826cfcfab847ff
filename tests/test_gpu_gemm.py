"""Variant (a) parity: the tcgen05 Q8 GEMM against the oracle.

Gate (north_star, see tests/gate.py): max error <= 2e-3 * RMS(y_exact) beyond
the final f16 rounding, where y_exact is the oracle's UNROUNDED (f64) result
over f16-dequantised weights (q8_gemm.metal:25-26 semantics) -- comparing two
f16-rounded results could exceed the gate from 1-ulp flips alone.  Every call
goes through the C ABI.
"""
import numpy as np
import pytest

from madi_b200 import synth

from tests.gate import check as gate_check

pytestmark = pytest.mark.gpu


def _t(a, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _check(y_gpu, y_exact, what):
    return gate_check(y_gpu.float().cpu().numpy(), y_exact, what, f16_out=True)


def _run(madi, oracle, M, N, K, epi, seed=1, bias_f16=False):
    from madi_b200 import q8
    qs, sc = synth.q8_weight(N, K, seed)
    x = synth.activations(M, K, seed + 100)
    b = synth.bias(N, seed + 200, np.float16 if bias_f16 else np.float32)
    r = synth.activations(M, N, seed + 300) if epi == q8.EPI_BIAS_RES else None
    W = q8.Q8Weight(_t(qs), _t(sc))
    y = q8.linear(W, _t(x), bias=_t(b) if epi != q8.EPI_NONE else None, epi=epi,
                  residual=_t(r) if r is not None else None)
    import torch
    torch.cuda.synchronize()
    y_exact = oracle.linear_f16(x, qs, sc, bias=b.astype(np.float32), epi=epi, residual=r)
    return _check(y, y_exact, f"M={M} N={N} K={K} epi={epi}")


@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_config0_shape_all_epilogues(madi, oracle, epi):
    # config 0: 1500 x 1280 x 1280 (M not a multiple of the token tile)
    _run(madi, oracle, 1500, 1280, 1280, epi)


@pytest.mark.parametrize("M", [17, 50, 129, 191, 192, 193, 385])
def test_token_tails(madi, oracle, M):
    # 17: the smallest M the tensor-core path takes for K % 256 == 0 (m <= 16 streams)
    _run(madi, oracle, M, 256, 256, 1, seed=M)


@pytest.mark.parametrize("N", [32, 96, 160, 1312])
def test_feature_tails(madi, oracle, N):
    # N not a multiple of the 128-row weight tile
    _run(madi, oracle, 200, N, 128, 2, seed=N)


@pytest.mark.parametrize("K", [32, 96, 160, 2080])
def test_odd_k_blocks(madi, oracle, K):
    # K % 64 == 32: the last pipeline stage is half filled
    _run(madi, oracle, 300, 256, K, 1, seed=K)


@pytest.mark.parametrize("epi", [0, 1, 2, 3])
@pytest.mark.parametrize("K", [320, 288])
def test_wide_pair_tile_ragged_waves(madi, oracle, epi, K):
    # M = 3001, N = 2560: 140 tiles of 224 tokens (two waves of 74 pairs, the last
    # tile 89 tokens) cost less than 160 tiles of 192 (three waves), so the launcher
    # picks the 224-token pair tile; K = 288 leaves the last stage half filled
    _run(madi, oracle, 3001, 2560, K, epi, seed=K + epi)


def test_bias_f16(madi, oracle):
    _run(madi, oracle, 257, 384, 320, 2, bias_f16=True)


def test_encoder_ffn_pair_b1(madi, oracle):
    """config 1, B=1: fc1 + bias + GELU -> H (f16), then fc2 + bias + residual(X)."""
    import torch
    from madi_b200 import q8
    w = synth.ffn_weights(3)
    x = synth.activations(1500, 1280, 77)
    W1 = q8.Q8Weight(_t(w["fc1_qs"]), _t(w["fc1_scales"]))
    W2 = q8.Q8Weight(_t(w["fc2_qs"]), _t(w["fc2_scales"]))
    X = _t(x)
    H = q8.linear(W1, X, bias=_t(w["fc1_bias"]), epi=q8.EPI_BIAS_GELU)
    Y = q8.linear(W2, H, bias=_t(w["fc2_bias"]), epi=q8.EPI_BIAS_RES, residual=X)
    torch.cuda.synchronize()
    h_exact = oracle.linear_f16(x, w["fc1_qs"], w["fc1_scales"], w["fc1_bias"], oracle.EPI_BIAS_GELU)
    _check(H, h_exact, "fc1")
    # fc2 checked on the GPU's own H (isolates the kernel) and end to end
    h16 = H.cpu().numpy()
    y_exact = oracle.linear_f16(h16, w["fc2_qs"], w["fc2_scales"], w["fc2_bias"], oracle.EPI_BIAS_RES, residual=x)
    _check(Y, y_exact, "fc2")
    y_chain = oracle.linear_f16(h_exact.astype(np.float16), w["fc2_qs"], w["fc2_scales"], w["fc2_bias"],
                                oracle.EPI_BIAS_RES, residual=x)
    _check(Y, y_chain, "ffn pair end to end")


def test_reference_names_through_dispatch(madi, oracle):
    """mul_mm_q8 / m4_gemm_q8tg / m4_gemm_q8_bias_gelu, called like the reference's
    test_q8gemm.zig: kernelParams-style argument arrays through madi_dispatch."""
    import torch
    from madi_b200 import backend as mtl
    M, N, K = 50, 64, 96     # test_q8gemm.zig:41 correctness shape (partial M tile)
    qs, sc = synth.q8_weight(N, K, 7)
    x = synth.activations(M, K, 8)
    b = synth.bias(N, 9)
    A, Q, S, Bb = _t(x), _t(qs), _t(sc), _t(b)
    C = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    f = mtl.get_function("mul_mm_q8")
    mtl.dispatch(f, ((N + 31) // 32, (M + 31) // 32, 1), (128, 1, 1),
                 [mtl.Arg.buf(C), mtl.Arg.buf(A), mtl.Arg.buf(Q), mtl.Arg.buf(S),
                  mtl.Arg.u32(M), mtl.Arg.u32(N), mtl.Arg.u32(K)])
    mtl.sync(10000)
    _check(C, oracle.linear_f16(x, qs, sc), "mul_mm_q8")
    # the reference's own (loose) gate, test_q8gemm.zig:71
    assert np.abs(C.float().cpu().numpy() - oracle.linear_f16(x, qs, sc)).max() <= 0.2
    for name, gelu in (("m4_gemm_q8tg", 0), ("m4_gemm_q8tg", 1), ("m4_gemm_q8_bias_gelu", 1)):
        C.zero_()
        mtl.dispatch(mtl.get_function(name), (1, 1, 1), (128, 1, 1),
                     [mtl.Arg.buf(A), mtl.Arg.buf(Q), mtl.Arg.buf(S), mtl.Arg.buf(C), mtl.Arg.buf(Bb),
                      mtl.Arg.u32(M), mtl.Arg.u32(N), mtl.Arg.u32(K), mtl.Arg.u32(gelu)])
        mtl.sync(10000)
        epi = oracle.EPI_BIAS_GELU if gelu else oracle.EPI_BIAS
        _check(C, oracle.linear_f16(x, qs, sc, b, epi), f"{name}(act_gelu={gelu})")


def test_deterministic_repeat(madi):
    import torch
    from madi_b200 import q8
    qs, sc = synth.q8_weight(1280, 1280, 5)
    W = q8.Q8Weight(_t(qs), _t(sc))
    X = _t(synth.activations(1500, 1280, 6))
    y1 = q8.linear(W, X)
    y2 = q8.linear(W, X)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("M,N", [(16, 6483), (64, 6483), (200, 1312), (160, 25933)])
def test_f32_output_without_epilogue(madi, oracle, M, N):
    """f32 y and no epilogue (a vocab-head shard over many token slots): f32
    accumulation written without rounding, so the error against the exact result
    is held to 1e-4 x RMS, far inside the gate.  Up to 16 rows the skinny GEMM
    runs it (exact int8 weights times f32 block scales, as gemv_q8 computes); above
    16 the tensor-core GEMM (weights dequantised to f16 first, as the encoder does)."""
    import torch
    from madi_b200 import q8
    K = 1280
    qs, sc = synth.q8_weight(N, K, M + N)
    x = synth.activations(M, K, M + N + 1)
    W = q8.Q8Weight(_t(qs), _t(sc))
    y = q8.linear(W, _t(x), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32
    if M <= 16:
        y_exact = oracle.gemv_q8(x.astype(np.float32), qs, sc)
    else:
        y_exact = oracle.linear_f16(x, qs, sc, epi=oracle.EPI_NONE)
    err = np.abs(y.cpu().numpy().astype(np.float64) - y_exact).max()
    rms = np.sqrt(np.mean(y_exact ** 2))
    assert err <= 1e-4 * rms, f"M={M} N={N}: max err {err:.3e} vs rms {rms:.3e}"


@pytest.mark.parametrize("M,N,K", [(1500, 1280, 1280), (3000, 1280, 5120), (333, 160, 96)])
def test_f32_residual_stream_epilogue(madi, oracle, M, N, K):
    """f32 out + BIAS_RES + f32 residual on the tensor-core path: the encoder's residual
    stream x += half(acc) + bias in place (the add of bias_res_ln_f16 moved into the
    GEMM).  x must equal (x + f16(acc)) + bias with the f16 rounding of the projection
    as the only approximation: max error beyond the half-ulp of the f16 projection
    <= 2e-3 x RMS(acc), under the shared gate's rule."""
    import torch
    from madi_b200 import q8
    from tests.gate import half_ulp16
    qs, sc = synth.q8_weight(N, K, M + K)
    a = synth.activations(M, K, M + 1)
    b = synth.bias(N, 4)
    x0 = np.random.default_rng(M).standard_normal((M, N)).astype(np.float32)
    X = _t(x0)
    q8.linear(q8.Q8Weight(_t(qs), _t(sc)), _t(a), bias=_t(b), epi=q8.EPI_BIAS_RES, residual=X, out=X)
    torch.cuda.synchronize()
    acc = oracle.linear_f16(a, qs, sc)
    want = x0.astype(np.float64) + acc + b.astype(np.float64)
    got = X.cpu().numpy().astype(np.float64)
    excess = np.maximum(np.abs(got - want) - half_ulp16(acc) - 1e-6 * np.abs(want), 0.0)
    rms = np.sqrt(np.mean(acc ** 2))
    assert excess.max() <= 2e-3 * rms, f"excess {excess.max() / rms:.3e} x RMS"
    # the add itself is exact f32 arithmetic on the f16-rounded projection of the GPU
    y16 = q8.linear(q8.Q8Weight(_t(qs), _t(sc)), _t(a))
    torch.cuda.synchronize()
    ref = (torch.from_numpy(x0) + y16.float().cpu()) + torch.from_numpy(b.astype(np.float32))
    assert torch.equal(X.cpu(), ref), "x != (x + f16 projection) + bias in f32"
