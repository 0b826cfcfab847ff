"""numpy front-end for the CPU baseline (oracle/cpu_baseline.c).

MEASUREMENT INFRASTRUCTURE ONLY: bench.py's cpu_baseline leg and its
`--impl reference` arm time the reference's CPU computation of the Q8 linear
(test_q8gemm.zig:59-69) through this module; madi_b200 never imports it.

The library is compiled on the host that runs it (-march=native) into
oracle/_build/native-<cpu key>/, the key a hash of the CPU model and feature
flags, so a build from another machine is never loaded.
"""
import ctypes
import hashlib
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
EPI_NONE, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RES = 0, 1, 2, 3

_lib = None


def cpu_key() -> str:
    model, flags = "", ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name") and not model:
                    model = line.split(":", 1)[1].strip()
                elif line.startswith("flags") and not flags:
                    flags = line.split(":", 1)[1].strip()
    except OSError:
        pass
    return hashlib.sha1((model + "|" + flags).encode()).hexdigest()[:12]


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def build() -> str:
    d = os.path.join("_build", "native-" + cpu_key())
    subprocess.run(["make", "-s", "-C", HERE, "native", f"NATIVE_DIR={d}"], check=True)
    return os.path.join(HERE, d, "libmadi_cpu_baseline.so")


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(build())
        P, I = ctypes.c_void_p, ctypes.c_int
        L.madi_cpu_linear_faithful.argtypes = [P, I, I, P, P, I, P, I, P, P]
        L.madi_cpu_dequant_f32.argtypes = [P, P, I, I, P, I]
        L.madi_cpu_linear_tiled.argtypes = [P, I, I, P, I, P, I, P, P, I]
        L.madi_cpu_gemv_q8.argtypes = [P, I, P, P, I, I, P, I, P, I]
        L.madi_cpu_threads.restype = I
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


def linear_faithful(X, qs, scales, bias=None, epi=EPI_NONE, residual=None):
    """test_q8gemm.zig:59-69 as written (one thread) + the m4_gemm epilogue -> f16 [M][N]."""
    X, qs, sc = _c(X, np.float16), _c(qs, np.int8), _c(scales, np.float16)
    M, K = X.shape
    N = qs.shape[0]
    y = np.empty((M, N), np.uint16)
    r = _c(residual, np.float16)
    lib().madi_cpu_linear_faithful(_p(X.view(np.uint16)), M, K, _p(qs), _p(sc.view(np.uint16)), N,
                                   _p(_c(bias, np.float32)), epi, None if r is None else _p(r.view(np.uint16)),
                                   _p(y))
    return y.view(np.float16)


def dequant_f32(qs, scales, nthreads):
    """f32 [N][K] = float(q) * float(s) (once per run)."""
    qs, sc = _c(qs, np.int8), _c(scales, np.float16)
    N, K = qs.shape
    w = np.empty((N, K), np.float32)
    lib().madi_cpu_dequant_f32(_p(qs), _p(sc.view(np.uint16)), N, K, _p(w), nthreads)
    return w


def linear_tiled(X, wdq, bias=None, epi=EPI_NONE, residual=None, nthreads=1, out=None):
    """The same sums on `nthreads` cores over pre-dequantised f32 weights -> f16 [M][N]."""
    X = _c(X, np.float16)
    M, K = X.shape
    N = wdq.shape[0]
    y = out if out is not None else np.empty((M, N), np.float16)
    r = _c(residual, np.float16)
    lib().madi_cpu_linear_tiled(_p(X.view(np.uint16)), M, K, _p(wdq), N, _p(_c(bias, np.float32)), epi,
                                None if r is None else _p(r.view(np.uint16)), _p(y.view(np.uint16)), nthreads)
    return y


def gemv_q8(x, qs, scales, bias=None, epi=EPI_NONE, y=None, nthreads=1):
    """Decode projection for M <= 16 f32 rows (int8 weights dequantised in registers)
    -> f32 [M][N]; with EPI_BIAS_RES, y holds the residual and is updated in place."""
    x = _c(x, np.float32)
    M, K = x.shape
    N = qs.shape[0]
    if y is None:
        y = np.zeros((M, N), np.float32)
    lib().madi_cpu_gemv_q8(_p(x), M, _p(qs), _p(scales.view(np.uint16)), N, K, _p(_c(bias, np.float32)), epi,
                           _p(y), nthreads)
    return y
