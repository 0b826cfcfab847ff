"""The whole large-v3-turbo-shaped encoder at its real depth -- 32 Q8 layers and
ln_post (madi_b200/encoder.py Encoder, the configuration-3 model) -- against the
same chain of the oracle's restatements, one chunk of 80 frames (a 160-frame mel) so
the f64 oracle runs in seconds.

The chain follows the reference's encoder (encoder.zig:235-315, encoder_ops.metal:
305-364) with its f16 rounding points: LN1 -> f16; QKV GEMM + bias -> f16; attention
-> f16; out-projection -> f16, added to the f32 residual with its bias; LN2 -> f16;
fc1 + bias + GELU -> f16; fc2 -> f16, added with its bias; after 32 layers ln_post.
The conv stem is f16 GEMMs through cuBLAS (not a Q8 op): the oracle starts from the
GPU's stem output.  Rounding points in series let the GPU and the oracle land an f16
ulp apart at any of them, and the residual stream carries that through 32 layers, so
the bars are on the whole output: max |err| <= 5e-2 x RMS and RMS(err) <= 5e-3 x RMS
(the one-layer test, tests/test_gpu_encoder_layer.py, holds each layer to 1e-2).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
FRAMES = 160


def _np(t):
    return t.detach().cpu().numpy()


def test_full_depth_encoder_against_oracle(madi, oracle):
    import torch
    from madi_b200 import encoder as enc, pipeline
    E = enc.Encoder(layers=32, seed=2)
    mel = torch.from_numpy(pipeline.synthetic_mel(1, first=11)[:, :, :FRAMES].copy()).cuda()
    seq = FRAMES // 2
    x0 = E.stem_all(mel)
    x = x0.clone()
    y = E.layers_forward(x, seq)
    torch.cuda.synchronize()

    h16 = lambda a: np.asarray(a, np.float64).astype(np.float16)
    D = enc.D
    xo = _np(x0).astype(np.float32)
    for L in E.layers:
        qkv_w = (_np(L.qkv.qs), _np(L.qkv.scales))
        _, yl = oracle.bias_res_ln(xo, None, None, _np(L.ln1[0]), _np(L.ln1[1]), enc.EPS)
        qkv = h16(oracle.linear_f16(h16(yl), *qkv_w, bias=_np(L.bqkv), epi=oracle.EPI_BIAS))
        a = h16(oracle.flash_attn_enc(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], enc.HEADS, seq))
        mo = h16(oracle.linear_f16(a, _np(L.o.qs), _np(L.o.scales)))
        xo, y2 = oracle.bias_res_ln(xo, mo, _np(L.bo), _np(L.ln2[0]), _np(L.ln2[1]), enc.EPS)
        hh = h16(oracle.linear_f16(h16(y2), _np(L.fc1.qs), _np(L.fc1.scales), bias=_np(L.b1),
                                   epi=oracle.EPI_BIAS_GELU))
        f = h16(oracle.linear_f16(hh, _np(L.fc2.qs), _np(L.fc2.scales)))
        xo = (xo + f.astype(np.float32)) + _np(L.b2).astype(np.float32)
    _, want = oracle.bias_res_ln(xo, None, None, _np(E.ln_post[0]), _np(E.ln_post[1]), enc.EPS)

    got = _np(y).astype(np.float64)
    rms = np.sqrt(np.mean(want ** 2))
    err = np.abs(got - want)
    print(f"32-layer encoder: max |err| {err.max() / rms:.3e} x RMS, RMS(err) {np.sqrt(np.mean(err ** 2)) / rms:.3e}"
          f" x RMS; residual stream {np.abs(_np(x) - xo).max() / np.sqrt(np.mean(xo.astype(np.float64) ** 2)):.3e}")
    assert np.isfinite(got).all()
    assert err.max() <= 5e-2 * rms, f"max |err| {err.max() / rms:.3e} x RMS"
    assert np.sqrt(np.mean(err ** 2)) <= 5e-3 * rms, f"RMS(err) {np.sqrt(np.mean(err ** 2)) / rms:.3e} x RMS"
