"""The one-CTA tcgen05 GEMM (selected with MADI_GEMM_PAIR=0; the CTA-pair kernel
is the default) against the same parity cases as test_gpu_gemm.py.  The switch
is read once per process, so the cases run in a child pytest process."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_single_cta_kernel_parity(madi):
    env = dict(os.environ, MADI_GEMM_PAIR="0")
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.join(HERE, "test_gpu_gemm.py"), "-q", "-x", "-m", "gpu",
                        "-p", "no:cacheprovider"],
                       cwd=os.path.dirname(HERE), env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
