"""Parity at the benchmarked configuration: BASELINE config 1, the encoder FFN
pair at B = 4 and B = 16 chunks (M = 6000 / 24000 frames), built exactly as
bench.py builds its timed step (synth.ffn_weights(0), X = synth.activations(M,
1280, 1000)), through the public API (madi_b200.q8.linear -> madi_q8_linear).

The oracle's f64 loop would need minutes for all 24000 rows, so a seeded sample
of 512 rows is checked, every one of its 5120 (fc1) / 1280 (fc2) columns, under
the shared gate (tests/gate.py: max error beyond the final f16 half-ulp <=
2e-3 x RMS of the exact result).  fc2 is checked on the GPU's own H rows (the
kernel in isolation) and end to end against the oracle's chain.  The sample
includes the first and last rows (the first and last token tiles) and rows at
the 192-token tile boundaries.  Across all rows the two GEMMs are checked for
size-independent properties: finite output everywhere, and each chunk's rows
equal to the same chunk computed alone (a row's result does not depend on M).
"""
import numpy as np
import pytest

from madi_b200 import synth

from tests.gate import check

pytestmark = pytest.mark.gpu
D, F, SEQ = 1280, 5120, 1500


def _t(a, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _sample_rows(M, n=512, seed=0):
    g = np.random.default_rng(seed + M)
    edges = [0, 1, 191, 192, 193, M // 2, M - 193, M - 192, M - 2, M - 1]
    rest = g.choice(M, size=n - len(edges), replace=False)
    return np.unique(np.concatenate([np.array(edges), rest]))[:n]


@pytest.mark.parametrize("B", [4, 16])
def test_ffn_pair_bench_config(madi, oracle, B):
    import torch
    from madi_b200 import q8
    M = B * SEQ
    w = synth.ffn_weights(0)
    x = synth.activations(M, D, 1000)
    W1 = q8.Q8Weight(_t(w["fc1_qs"]), _t(w["fc1_scales"]))
    W2 = q8.Q8Weight(_t(w["fc2_qs"]), _t(w["fc2_scales"]))
    b1, b2 = _t(w["fc1_bias"]), _t(w["fc2_bias"])
    X = _t(x)
    H = q8.linear(W1, X, bias=b1, epi=q8.EPI_BIAS_GELU)
    Y = q8.linear(W2, H, bias=b2, epi=q8.EPI_BIAS_RES, residual=X)
    torch.cuda.synchronize()
    assert torch.isfinite(H).all() and torch.isfinite(Y).all()

    rows = _sample_rows(M)
    xs = x[rows]
    h_exact = oracle.linear_f16(xs, w["fc1_qs"], w["fc1_scales"], w["fc1_bias"], oracle.EPI_BIAS_GELU)
    ex1, raw1 = check(H[rows].float().cpu().numpy(), h_exact, f"fc1 B={B}", f16_out=True)
    h_gpu = H[rows].cpu().numpy()
    y_exact = oracle.linear_f16(h_gpu, w["fc2_qs"], w["fc2_scales"], w["fc2_bias"], oracle.EPI_BIAS_RES,
                                residual=xs)
    ex2, raw2 = check(Y[rows].float().cpu().numpy(), y_exact, f"fc2 B={B}", f16_out=True)
    y_chain = oracle.linear_f16(h_exact.astype(np.float16), w["fc2_qs"], w["fc2_scales"], w["fc2_bias"],
                                oracle.EPI_BIAS_RES, residual=xs)
    ex3, raw3 = check(Y[rows].float().cpu().numpy(), y_chain, f"ffn pair B={B} end to end", f16_out=True)
    print(f"B={B} M={M} rows={rows.size}: fc1 raw {raw1:.2e} excess {ex1:.2e}; fc2 raw {raw2:.2e} excess {ex2:.2e};"
          f" chain raw {raw3:.2e} excess {ex3:.2e}")

    # a chunk computed alone gives the same rows as inside the M-row batch
    for c in (0, B - 1):
        Xc = X[c * SEQ:(c + 1) * SEQ].contiguous()
        Hc = q8.linear(W1, Xc, bias=b1, epi=q8.EPI_BIAS_GELU)
        Yc = q8.linear(W2, Hc, bias=b2, epi=q8.EPI_BIAS_RES, residual=Xc)
        torch.cuda.synchronize()
        assert torch.equal(Hc, H[c * SEQ:(c + 1) * SEQ]), f"chunk {c}: fc1 rows depend on M"
        assert torch.equal(Yc, Y[c * SEQ:(c + 1) * SEQ]), f"chunk {c}: fc2 rows depend on M"
