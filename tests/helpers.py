"""Shared checks for the parity tests."""
from __future__ import annotations

import numpy as np

# Tolerance stated by the north star for fp32 output: relative Frobenius error
# <= 1e-5 and per-element |err| <= 1e-3 * ||oracle row||_2 (the row norm is
# taken over the oracle's output row D[i, :]).
FROB_TOL_F32 = 1e-5
ROW_TOL = 1e-3
# bf16 output: the stored value is the fp32 result rounded to bf16, which adds
# at most 2^-8 relative error per element (2^-9 for round-to-nearest) on top
# of the fp32 tolerance.
BF16_REL = 2.0 ** -8


def check_gemm(got: np.ndarray, ref: np.ndarray, bf16: bool = False) -> dict:
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    assert got.shape == ref.shape
    assert np.isfinite(got).all(), "non-finite output"
    err = got - ref
    frob = np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30)
    row_norm = np.linalg.norm(ref, axis=1, keepdims=True)
    elem_tol = ROW_TOL * row_norm
    if bf16:
        elem_tol = elem_tol + BF16_REL * np.abs(ref)
        frob_tol = FROB_TOL_F32 + BF16_REL
    else:
        frob_tol = FROB_TOL_F32
    worst = float(np.max(np.abs(err) - elem_tol))
    info = {"frob": float(frob), "worst_excess": worst, "max_abs": float(np.max(np.abs(err)))}
    assert frob <= frob_tol, f"relative Frobenius {frob:.3e} > {frob_tol:.1e} ({info})"
    assert worst <= 0.0, f"per-element tolerance exceeded ({info})"
    return info
