"""Shared helpers for the parity tests.

Relative error used throughout: max-norm ratio  max|a - b| / max|b|  over the
whole tensor (b = oracle).  Bars (north star): 2e-3 for f32-accumulation paths,
3e-2 where bf16 tensor-core prefill is used.  Index/placement checks are exact.
"""
import numpy as np

TOL_F32 = 2e-3
TOL_BF16 = 3e-2


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.abs(b).max()
    return float(np.abs(a - b).max() / (den if den > 0 else 1.0))


def assert_close(a, b, tol, what=""):
    e = rel_err(a, b)
    assert np.all(np.isfinite(a)), f"{what}: non-finite values"
    assert e <= tol, f"{what}: rel err {e:.3e} > {tol:.1e}"
    return e
