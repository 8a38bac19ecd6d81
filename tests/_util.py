"""Shared helpers for the parity tests.

Every comparison checks two relative errors against the same bar:
  * max-norm ratio   max|a - b| / max|b|  over the whole tensor (b = oracle);
  * elementwise      max |a - b| / |b|    over the elements with |b| >= FLOOR * max|b|.
The floor keeps the elementwise check away from elements that are tiny next to
the tensor's scale, where a relative error says nothing about the arithmetic.
Bars (north star): 2e-3 for f32-accumulation paths, 3e-2 where bf16
tensor-core prefill is used.  Index / placement checks are exact.

Floors: 1% of max|ref| for the f32 paths.  The bf16 attention prefill rounds
the softmax weights P to bf16 (2^-9 relative) before P V; an output element at
1% of the tensor's scale then carries ~100x that relative error (measured
~15%), so its elementwise check uses a 10% floor (measured ~2e-2 there, with
the max-norm error ~3e-3).
"""
import numpy as np

TOL_F32 = 2e-3
TOL_BF16 = 3e-2
FLOOR = 1e-2
FLOOR_BF16 = 1e-1


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.abs(b).max()
    return float(np.abs(a - b).max() / (den if den > 0 else 1.0))


def rel_err_elem(a, b, floor=FLOOR):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    scale = np.abs(b).max()
    if scale == 0:
        return float(np.abs(a).max())
    big = np.abs(b) >= floor * scale
    return float((np.abs(a - b)[big] / np.abs(b)[big]).max())


def assert_close(a, b, tol, what="", floor=None, elem_tol=None):
    """Max-norm and elementwise (above floor * max|b|) relative error <= tol
    (elem_tol if given); returns the max-norm error.  The floor defaults to
    FLOOR_BF16 for the bf16 bar and FLOOR otherwise."""
    if floor is None:
        floor = FLOOR_BF16 if tol >= TOL_BF16 else FLOOR
    assert np.all(np.isfinite(a)), f"{what}: non-finite values"
    e = rel_err(a, b)
    assert e <= tol, f"{what}: max-norm rel err {e:.3e} > {tol:.1e}"
    ee = rel_err_elem(a, b, floor)
    et = tol if elem_tol is None else elem_tol
    assert ee <= et, f"{what}: elementwise rel err {ee:.3e} > {et:.1e} (|ref| >= {floor:g} max|ref|)"
    return e
