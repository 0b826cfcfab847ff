"""Parity of the encoder's residual + LayerNorm step beside the Q8 linear
(bias_res_ln_f16 / layer_norm_f16, encoder_ops.metal:305-364) against the oracle.

The f32 residual stream x must match the reference's update bit for bit
((x + float(mo)) + bias); the f16 output passes the shared gate (tests/gate.py)
against the oracle's unrounded LayerNorm.
"""
import numpy as np
import pytest

from tests.gate import check as gate_check

pytestmark = pytest.mark.gpu


def _t(a, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _inputs(rows, d, seed):
    g = np.random.default_rng(seed)
    x = g.standard_normal((rows, d)).astype(np.float32) * 3.0 + 0.5
    mo = g.standard_normal((rows, d)).astype(np.float16)
    b = (g.standard_normal(d) * 0.02).astype(np.float32)
    gamma = (1.0 + 0.1 * g.standard_normal(d)).astype(np.float32)
    beta = (0.1 * g.standard_normal(d)).astype(np.float32)
    return x, mo, b, gamma, beta


@pytest.mark.parametrize("rows,d", [(1, 1280), (7, 1280), (1500, 1280), (333, 128), (64, 2048), (24000, 1280)])
def test_bias_res_ln(madi, oracle, rows, d):
    from madi_b200 import q8
    x, mo, b, gamma, beta = _inputs(rows, d, rows + d)
    X = _t(x)
    y = q8.bias_res_ln_f16(X, _t(mo), _t(b), _t(gamma), _t(beta), eps=1e-5)
    import torch
    torch.cuda.synchronize()
    x_ex, y_ex = oracle.bias_res_ln(x, mo, b, gamma, beta, 1e-5)
    assert np.array_equal(X.cpu().numpy(), x_ex), "residual stream differs from the reference's f32 update"
    gate_check(y.float().cpu().numpy(), y_ex, f"bias_res_ln rows={rows} d={d}", f16_out=True)


@pytest.mark.parametrize("rows,d", [(3, 1280), (1500, 1280), (17, 384)])
def test_layer_norm(madi, oracle, rows, d):
    from madi_b200 import q8
    import torch
    x, _, _, gamma, beta = _inputs(rows, d, 5 * rows + d)
    X = _t(x)
    y = q8.layer_norm_f16(X, _t(gamma), _t(beta), eps=1e-6)
    torch.cuda.synchronize()
    x_ex, y_ex = oracle.bias_res_ln(x, None, None, gamma, beta, 1e-6)
    assert np.array_equal(X.cpu().numpy(), x), "layer_norm_f16 must not modify x"
    gate_check(y.float().cpu().numpy(), y_ex, f"layer_norm rows={rows} d={d}", f16_out=True)


def test_by_name_with_reference_grid(madi, oracle):
    """bias_res_ln_f16 / layer_norm_f16 by name: the reference's argument orders,
    the row count taken from grid x (Grid=(rows) Block=256, encoder_ops.metal:304)."""
    import torch
    from madi_b200 import backend as mtl
    rows, d = 40, 1280
    x, mo, b, gamma, beta = _inputs(rows, d, 77)
    X, Y = _t(x), torch.empty((rows, d), dtype=torch.float16, device="cuda")
    mtl.dispatch(mtl.get_function("bias_res_ln_f16"), (rows, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(X), mtl.Arg.buf(_t(mo)), mtl.Arg.buf(_t(b)), mtl.Arg.buf(Y), mtl.Arg.buf(_t(gamma)),
                  mtl.Arg.buf(_t(beta)), mtl.Arg.u32(d), mtl.Arg.f32(1e-5)])
    mtl.sync(10000)
    x_ex, y_ex = oracle.bias_res_ln(x, mo, b, gamma, beta, 1e-5)
    assert np.array_equal(X.cpu().numpy(), x_ex)
    gate_check(Y.float().cpu().numpy(), y_ex, "bias_res_ln_f16 by name", f16_out=True)
    Y2 = torch.empty_like(Y)
    mtl.dispatch(mtl.get_function("layer_norm_f16"), (rows, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(X), mtl.Arg.buf(Y2), mtl.Arg.buf(_t(gamma)), mtl.Arg.buf(_t(beta)), mtl.Arg.u32(d),
                  mtl.Arg.f32(1e-5)])
    mtl.sync(10000)
    _, y2_ex = oracle.bias_res_ln(x_ex, None, None, gamma, beta, 1e-5)
    gate_check(Y2.float().cpu().numpy(), y2_ex, "layer_norm_f16 by name", f16_out=True)


def test_rejects_unsupported_widths(madi):
    import torch
    from madi_b200 import q8
    from madi_b200._lib import MadiError, MADI_EINVAL
    for d in (96, 1000, 4096):
        x = torch.zeros((4, d), dtype=torch.float32, device="cuda")
        g = torch.ones(d, dtype=torch.float32, device="cuda")
        with pytest.raises(MadiError) as e:
            q8.layer_norm_f16(x, g, g)
        assert e.value.code == MADI_EINVAL


@pytest.mark.parametrize("rows,d", [(1, 1280), (8, 1280), (300, 384)])
def test_decoder_f32_forms(madi, oracle, rows, d):
    """bias_res_ln / layer_norm (encoder_ops.metal:14-120): f32 MO and f32 Y, typed
    and by name; the residual stream bit-exact, Y within 1e-5 x max|Y|."""
    import torch
    from madi_b200 import q8
    from madi_b200 import backend as mtl
    g = np.random.default_rng(rows + d)
    x = (g.standard_normal((rows, d)) * 3.0).astype(np.float32)
    mo = g.standard_normal((rows, d)).astype(np.float32)
    b = (g.standard_normal(d) * 0.02).astype(np.float32)
    gamma = (1.0 + 0.1 * g.standard_normal(d)).astype(np.float32)
    beta = (0.1 * g.standard_normal(d)).astype(np.float32)
    X = _t(x)
    y = q8.bias_res_ln(X, _t(mo), _t(b), _t(gamma), _t(beta), eps=1e-5)
    torch.cuda.synchronize()
    x_ex, y_ex = oracle.bias_res_ln_f32(x, mo, b, gamma, beta, 1e-5)
    assert np.array_equal(X.cpu().numpy(), x_ex)
    assert np.abs(y.cpu().numpy() - y_ex).max() <= 1e-5 * np.abs(y_ex).max()
    Y2 = torch.empty((rows, d), dtype=torch.float32, device="cuda")
    mtl.dispatch(mtl.get_function("layer_norm"), (rows, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(X), mtl.Arg.buf(Y2), mtl.Arg.buf(_t(gamma)), mtl.Arg.buf(_t(beta)), mtl.Arg.u32(d),
                  mtl.Arg.f32(1e-5)])
    mtl.sync(10000)
    _, y2_ex = oracle.bias_res_ln_f32(x_ex, None, None, gamma, beta, 1e-5)
    assert np.abs(Y2.cpu().numpy() - y2_ex).max() <= 1e-5 * np.abs(y2_ex).max()
    X3 = _t(x)
    Y3 = torch.empty((rows, d), dtype=torch.float32, device="cuda")
    mtl.dispatch(mtl.get_function("bias_res_ln"), (rows, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(X3), mtl.Arg.buf(_t(mo)), mtl.Arg.buf(_t(b)), mtl.Arg.buf(Y3), mtl.Arg.buf(_t(gamma)),
                  mtl.Arg.buf(_t(beta)), mtl.Arg.u32(d), mtl.Arg.f32(1e-5)])
    mtl.sync(10000)
    assert np.array_equal(X3.cpu().numpy(), x_ex)
    assert np.abs(Y3.cpu().numpy() - y_ex).max() <= 1e-5 * np.abs(y_ex).max()
