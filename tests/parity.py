"""Parity metric shared by the GPU tests.

Per tensor: max|a - e| <= tol * (max|e| + eps), plus elementwise
|a - e| <= tol * (1 + |e|) (the convention of sheaf/tests/prng_tests.rs:43-62).
tol = 1e-5 for fp32, 2e-2 for bf16; gathered rows / indices are compared
bit-exactly elsewhere.
"""
import numpy as np

TOL_F32 = 1e-5
TOL_BF16 = 2e-2


def assert_close(actual, expected, tol, name="", eps=1e-30, sum_abs=None):
    """sum_abs (optional, per element): the sum of the absolute values of the
    terms an output element sums. Its f32 rounding (a few ulps of that sum,
    4 * 2^-24 * sum_abs) is added to the elementwise bound: a long f32 sum
    whose exact value is near zero carries the rounding of its large partial
    sums, whatever order it is summed in."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, f"{name}: shape {a.shape} != {e.shape}"
    assert np.isfinite(a).all(), f"{name}: non-finite values"
    err = np.abs(a - e)
    scale = np.abs(e).max(initial=0.0)
    worst = err.max(initial=0.0)
    assert worst <= tol * (scale + eps), f"{name}: max err {worst:.3e} > {tol:g} * max|e| {scale:.3e}"
    bound = tol * (1.0 + np.abs(e))
    if sum_abs is not None:
        bound = bound + 4.0 * 2.0 ** -24 * np.asarray(sum_abs, np.float64)
    assert (err <= bound).all(), f"{name}: elementwise bound violated"


def rel_err(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return float(np.abs(a - e).max(initial=0.0) / max(np.abs(e).max(initial=0.0), 1e-30))
