"""The parity gate shared by the GPU tests.

north_star: outputs within max |err| <= 2e-3 x output RMS, against the
oracle's unrounded (f64) result.  For f16 outputs the last rounding to f16 is
part of the output format, not of the computation: a correctly rounded f16 of
the exact value may already sit half an f16 ulp away, which at Gaussian tails
(|y| ~ 5 RMS) is up to ~2.4e-3 RMS by itself.  So for f16 outputs the gate
applies to the error BEYOND that half ulp:
    excess_i = max(0, |y_i - exact_i| - ulp16(exact_i) / 2)
    max(excess) <= 2e-3 * RMS(exact)
For f32 outputs excess_i = |y_i - exact_i|.  The raw ratio is returned too.
"""
import numpy as np

TOL = 2e-3


def half_ulp16(v: np.ndarray) -> np.ndarray:
    a = np.abs(v).astype(np.float64)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -14)))      # subnormal range has the 2^-24 spacing
    return np.ldexp(1.0, (e - 10).astype(np.int64)) / 2


def check(y, exact, what: str, f16_out: bool, tol: float = TOL):
    y = np.asarray(y, dtype=np.float64).reshape(exact.shape)
    assert np.isfinite(y).all(), f"{what}: non-finite output"
    rms = float(np.sqrt(np.mean(exact ** 2)))
    diff = np.abs(y - exact)
    excess = np.maximum(diff - half_ulp16(exact), 0.0) if f16_out else diff
    raw = float(diff.max()) / rms
    ex = float(excess.max()) / rms
    assert ex <= tol, f"{what}: max excess error {ex:.3e} x RMS > {tol} (raw max|err| {raw:.3e} x RMS)"
    return ex, raw
