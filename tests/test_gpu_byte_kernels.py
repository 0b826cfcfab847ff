"""The two byte/integer kernels beside the linear, bit for bit on the GPU:

* dequant_q8_f16 (q8_gemm.metal:12-27, the reference's kDeq, encoder.zig:262-270):
  f16 [K][N] = half(float(q) * float(s)), transposed -- called by name through
  madi_dispatch with the reference's argument order, and through the typed entry
  madi_q8_dequant_f16; both must equal the oracle's restatement exactly.
* quantInto on the device (madi_q8_quantize_f16; transcribe.zig:309-327,
  quantize_q8.py:27-40): every case of tests/golden/quant_q8_golden.npz -- the
  outputs of the reference's own quantize_q8.py on normal, wide-range and edge
  blocks (all-zero, single non-zero, exact .5 ties, f16 subnormals, +-65504) --
  must come back bit-identical, int8 quants and f16 scales alike.
"""
import os

import numpy as np
import pytest

from madi_b200 import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "quant_q8_golden.npz")


def _t(a, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


# (N, K): square, the FFN shapes, N not a multiple of the 64-row tile or of 8 (the
# scalar store path), the smallest K, K not a multiple of the 64-wide tile
DEQ_SHAPES = [(1280, 1280), (5120, 1280), (1280, 5120), (200, 96), (37, 32), (1000, 160), (51866 // 8, 1280)]


@pytest.mark.parametrize("N,K", DEQ_SHAPES)
def test_dequant_typed_bit_exact(madi, oracle, N, K):
    import torch
    from madi_b200 import q8
    qs, sc = synth.q8_weight(N, K, N + K)
    out = q8.dequant_f16(q8.Q8Weight(_t(qs), _t(sc)))
    torch.cuda.synchronize()
    assert tuple(out.shape) == (K, N)
    want = oracle.dequant_q8_f16(qs, sc)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("N,K", [(1280, 1280), (200, 96), (37, 32)])
def test_dequant_by_name_bit_exact(madi, oracle, N, K):
    """dequant_q8_f16(out, qs, scales, N, K) through madi_dispatch, as encoder.zig's
    kDeq calls it; the host grid is the reference's and is ignored."""
    import torch
    from madi_b200 import backend as mtl
    qs, sc = synth.q8_weight(N, K, 3 * N + K)
    out = torch.full((K, N), float("nan"), dtype=torch.float16, device="cuda")
    f = mtl.get_function("dequant_q8_f16")
    mtl.dispatch(f, ((N + 15) // 16, (K + 15) // 16, 1), (16, 16, 1),
                 [mtl.Arg.buf(out), mtl.Arg.buf(_t(qs)), mtl.Arg.buf(_t(sc)), mtl.Arg.u32(N), mtl.Arg.u32(K)])
    mtl.sync(10000)
    want = oracle.dequant_q8_f16(qs, sc)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_dequant_extreme_scales(madi, oracle):
    """Scales at the f16 extremes: products that overflow to inf, fall into the
    subnormal range or round to zero must round exactly as half(float(q)*float(s))."""
    import torch
    from madi_b200 import q8
    N, K = 64, 64
    g = np.random.default_rng(11)
    qs = g.integers(-127, 128, (N, K), dtype=np.int8)
    qs[0, :8] = [127, -127, 1, -1, 0, 64, -64, 3]
    pool = np.array([65504.0, 1024.0, 600.0, 6.1e-5, 6e-8, 1e-7, 2.0 ** -24, 0.0, 1.0, 0.5],
                    np.float32).astype(np.float16)
    sc = pool[g.integers(0, pool.size, (N, K // 32))]
    out = q8.dequant_f16(q8.Q8Weight(_t(qs), _t(sc)))
    torch.cuda.synchronize()
    want = oracle.dequant_q8_f16(qs, sc)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("case", ["normal", "wide", "edges"])
def test_device_quantiser_matches_reference_golden(madi, case):
    import torch
    from madi_b200 import q8
    g = np.load(GOLDEN)
    w = g[f"{case}_w_f16"].view(np.float16)
    W = q8.quantize_f16(_t(w))
    torch.cuda.synchronize()
    assert np.array_equal(W.qs.cpu().numpy(), g[f"{case}_qs"]), "int8 quants differ from quantize_q8.py"
    assert np.array_equal(W.scales.cpu().numpy().view(np.uint16), g[f"{case}_scales_f16"]), \
        "f16 scales differ from quantize_q8.py"


def test_device_quantiser_into_rows_of_stacked_weight(madi):
    """quantize_f16_into writes a row range of a larger weight (quantInto's row
    offset, transcribe.zig:309) and leaves the other rows untouched."""
    import torch
    from madi_b200 import q8
    g = np.load(GOLDEN)
    w = g["normal_w_f16"].view(np.float16)                     # [48][256]
    rows, dim = w.shape
    qs = torch.full((3 * rows, dim), 99, dtype=torch.int8, device="cuda")
    sc = torch.full((3 * rows, dim // 32), 7.0, dtype=torch.float16, device="cuda")
    q8.quantize_f16_into(_t(w), qs[rows:2 * rows], sc[rows:2 * rows])
    torch.cuda.synchronize()
    assert np.array_equal(qs[rows:2 * rows].cpu().numpy(), g["normal_qs"])
    assert np.array_equal(sc[rows:2 * rows].cpu().numpy().view(np.uint16), g["normal_scales_f16"])
    assert (qs[:rows] == 99).all() and (qs[2 * rows:] == 99).all()
    assert (sc[:rows] == 7.0).all() and (sc[2 * rows:] == 7.0).all()
