"""One Whisper-shaped encoder layer (madi_b200/encoder.py: f16 LayerNorms, tcgen05 Q8
QKV / out / fc1 / fc2 GEMMs with fused epilogues, tcgen05 flash attention) against the
same composition of the oracle's restatements, rounded to f16 at the same points
(layer-level parity on 2 chunks of 300 frames; every kernel also has its own test).

Bars: the f32 residual stream and the fc2 output within 1e-2 x RMS (f16 rounding
points in series, each of which may land one ulp apart: a one-ulp difference in the
attention output moves the f16 out-projection by a few ulps, which the residual
stream then carries).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _t(a, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_encoder_layer_composition(madi, oracle):
    import torch
    from madi_b200 import encoder as enc
    seq, chunks, D = 300, 2, enc.D
    w = enc.host_layer(seed=3)
    layer = enc.EncoderLayer(w)
    g = np.random.default_rng(8)
    x = g.standard_normal((chunks * seq, D)).astype(np.float32)
    prev_f = (g.standard_normal((chunks * seq, D)) * 0.5).astype(np.float16)
    prev_b2 = (g.standard_normal(D) * 0.02).astype(np.float32)
    X = _t(x)
    f = layer.forward(X, _t(prev_f), _t(prev_b2), seq=seq)
    torch.cuda.synchronize()

    h16 = lambda a: np.asarray(a, np.float64).astype(np.float16)
    x1, y = oracle.bias_res_ln(x, prev_f, prev_b2, *w["ln1"], enc.EPS)
    qkv = h16(oracle.linear_f16(h16(y), *w["qkv"], bias=w["bqkv"], epi=oracle.EPI_BIAS))
    a = h16(oracle.flash_attn_enc(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], enc.HEADS, seq))
    mo = h16(oracle.linear_f16(a, *w["o"]))
    x2, y2 = oracle.bias_res_ln(x1, mo, w["bo"], *w["ln2"], enc.EPS)
    hh = h16(oracle.linear_f16(h16(y2), *w["fc1"], bias=w["b1"], epi=oracle.EPI_BIAS_GELU))
    f_exact = oracle.linear_f16(hh, *w["fc2"])

    xr = X.cpu().numpy()
    xrms = np.sqrt(np.mean(x2.astype(np.float64) ** 2))
    assert np.abs(xr - x2).max() <= 1e-2 * xrms, f"residual: {np.abs(xr - x2).max() / xrms:.3e} x RMS"
    fr = f.float().cpu().numpy()
    rms = np.sqrt(np.mean(f_exact ** 2))
    assert np.abs(fr - f_exact).max() <= 1e-2 * rms, f"fc2 output: {np.abs(fr - f_exact).max() / rms:.3e} x RMS"


def test_fused_residual_layer_equals_separate_kernels(madi):
    """forward_fused (residual adds in the out-projection / fc2 epilogues, plain
    LayerNorms) against forward + bias_res_ln_f16: the residual stream and the
    LayerNorm outputs bit for bit, over two chained layers and ln_post; and the
    whole Encoder (stem, 2 layers, ln_post) the same in both modes."""
    import torch
    from madi_b200 import encoder as enc, pipeline, q8
    seq, chunks, D = 300, 2, enc.D
    L1, L2 = enc.EncoderLayer(enc.host_layer(seed=4)), enc.EncoderLayer(enc.host_layer(seed=5))
    g = np.random.default_rng(9)
    x = g.standard_normal((chunks * seq, D)).astype(np.float32)
    xa, xb = _t(x), _t(x)
    f1 = L1.forward(xa, None, None, seq=seq)
    f2 = L2.forward(xa, f1, L1.b2, seq=seq)
    ya = q8.bias_res_ln_f16(xa, f2, L2.b2, *L1.ln1, eps=enc.EPS)
    L1.forward_fused(xb, seq=seq)
    L2.forward_fused(xb, seq=seq)
    yb = q8.layer_norm_f16(xb, *L1.ln1, eps=enc.EPS)
    torch.cuda.synchronize()
    assert torch.equal(xa, xb), "residual stream differs"
    assert torch.equal(ya, yb), "LayerNorm output differs"
    mel = torch.from_numpy(pipeline.synthetic_mel(1, first=3)).cuda()
    outs = [enc.Encoder(layers=2, seed=6, fuse_res=f).forward(mel) for f in (True, False)]
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]), "encoder states differ between the fused and separate forms"


def test_encoder_graph_replay_equals_eager(madi):
    """Encoder.forward replays one CUDA graph per batch shape; its states equal the
    eager launches' bit for bit, on the capturing call and on a later replay with
    other input, and each call returns its own tensor."""
    import torch
    from madi_b200 import encoder as enc, pipeline
    eg = enc.Encoder(layers=2, seed=7, graphs=True)
    ee = enc.Encoder(layers=2, seed=7, graphs=False)
    m1 = torch.from_numpy(pipeline.synthetic_mel(2, first=21)[:, :, :320].copy()).cuda()
    m2 = torch.from_numpy(pipeline.synthetic_mel(2, first=40)[:, :, :320].copy()).cuda()
    a1, a2 = eg.forward(m1), eg.forward(m2)
    b1, b2 = ee.forward(m1), ee.forward(m2)
    torch.cuda.synchronize()
    assert torch.equal(a1, b1) and torch.equal(a2, b2), "graph replay differs from the eager pass"
    assert a1.data_ptr() != a2.data_ptr() and not torch.equal(a1, a2)
