"""The decode skinny GEMM has two kernels for K % 256 == 0: the row-unit kernel
(q8_gemv_rows.cu, the default for K <= 1280) and the tile kernel (q8_gemv_tile.cu,
K > 1280 and the fallback).  The choice is made once per process
(MADI_GEMV_ROWS=0 turns the row-unit kernel off), so this test runs the decoder's
K = 1280 shapes in a child process with MADI_GEMV_ROWS=0 -- the tile kernel --
and holds them to the same oracle bars as tests/test_gpu_gemv.py: the shared gate
and, for f32 in / out, 5e-5 x RMS.  It also checks that the two kernels give the
same greedy tokens on a 12-row head (both are f32-semantics sums; their block
orders differ, so values may differ in the last bits)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import numpy as np, torch
import madi_b200
from madi_b200 import q8, synth
from oracle import oracle
from tests.gate import check
madi_b200.init(0)
oracle.build()
t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
worst = 0.0
for (N, K, M, xdt, epi) in [(3840, 1280, 8, np.float32, 0), (1280, 1280, 3, np.float32, 1), (5120, 1280, 8, np.float16, 2),
                            (1280, 1280, 15, np.float16, 0), (51866, 1280, 8, np.float16, 0), (1280, 1280, 1, np.float32, 3)]:
    qs, sc = synth.q8_weight(N, K, N + M)
    x = synth.activations(M, K, M + 5, dtype=xdt)
    b = synth.bias(N, 9)
    res = synth.activations(M, N, 4, dtype=np.float32) if epi == 3 else None
    out = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    if res is not None:
        out.copy_(t(res))
    q8.linear(q8.Q8Weight(t(qs), t(sc)), t(x), bias=t(b) if epi else None, epi=epi,
              residual=out if res is not None else None, out=out)
    torch.cuda.synchronize()
    ex = oracle.gemv_q8(x.astype(np.float32), qs, sc, bias=b, epi=epi, res_in=res)
    _, raw = check(out.cpu().numpy(), ex, f"N={N} K={K} M={M}", f16_out=False)
    if xdt == np.float32:
        assert raw <= 5e-5, (N, K, M, raw)
    worst = max(worst, raw)
qs, sc = synth.q8_weight(51866, 1280, 77)
x = synth.activations(12, 1280, 78, dtype=np.float32)
lg = q8.linear(q8.Q8Weight(t(qs), t(sc)), t(x), x_round16=True)
tok = lg.argmax(dim=1).cpu().numpy()
np.save(OUT, tok)
print("worst", worst)
'''


def _run(rows: str, out: str):
    env = dict(os.environ, MADI_GEMV_ROWS=rows)
    code = f"OUT = {out!r}\n" + CHILD
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, f"MADI_GEMV_ROWS={rows}:\n{r.stdout[-2000:]}\n{r.stderr[-4000:]}"


def test_tile_kernel_parity_and_same_tokens(madi, tmp_path):
    import numpy as np
    a, b = str(tmp_path / "tile.npy"), str(tmp_path / "rows.npy")
    _run("0", a)
    _run("1", b)
    assert np.array_equal(np.load(a), np.load(b))
