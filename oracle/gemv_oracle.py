"""TEST INFRASTRUCTURE ONLY (checker, never the product path).

numpy restatement of the reference's dense GEMV contract:
  gemv_ref      cudalab/operators/gemv.py:192-201 (fp16: fp16(fp32 mv); fp32: mv)
  arith gate    cudalab/gemv_correctness.py:59-73,125-143,163-191
                (2 roundings per term, TOL_K = 2, ulp on the element grid)
Parity pinned by tests/golden/gemv_golden.npz (reference outputs).
"""
from __future__ import annotations

import numpy as np

TOL_K = 2.0
ROUNDINGS = 2.0
U = 2.0 ** -24


def exact_and_S(W: np.ndarray, x: np.ndarray):
    """fp64 exact GEMV of the stored values and S_n = sum_k |W x|."""
    wd = W.astype(np.float64)
    xd = x.astype(np.float64)
    return wd @ xd, np.abs(wd) @ np.abs(xd)


def ref_fp32(W: np.ndarray, x: np.ndarray) -> np.ndarray:
    """The reference result's arithmetic: fp32 products and sums, then the
    element type (row order of the sums is numpy's, which the gate allows)."""
    y = W.astype(np.float32) @ x.astype(np.float32)
    return y.astype(W.dtype)


def ulp(v: np.ndarray, dtype) -> np.ndarray:
    if np.dtype(dtype) == np.float32:
        vf = v.astype(np.float32)
        return (np.nextafter(vf, np.float32(np.inf)) - vf).astype(np.float64)
    a = np.abs(v.astype(np.float16).astype(np.float64))
    _, e = np.frexp(np.maximum(a, 2.0 ** -14))
    u = np.ldexp(1.0, e - 11)
    return np.where(a >= 2.0 ** -14, u, 2.0 ** -24)


def arith_ratio(y: np.ndarray, K: int, exact: np.ndarray, S: np.ndarray, dtype) -> float:
    yd = y.astype(np.float64)
    tol = TOL_K * (ROUNDINGS * K * U * S + 0.5 * ulp(yd, dtype) + 0.5 * ulp(exact, dtype))
    with np.errstate(invalid="ignore", divide="ignore"):
        r = np.abs(yd - exact) / tol
    r = np.where(np.isfinite(r), r, 0.0)
    return float(r.max()) if r.size else 0.0


def check(y: np.ndarray, W: np.ndarray, x: np.ndarray) -> dict:
    ex, S = exact_and_S(W, x)
    ratio = arith_ratio(y, W.shape[1], ex, S, W.dtype)
    finite = bool(np.isfinite(y.astype(np.float64)).all())
    return {"arith_max_ratio": ratio, "finite": finite, "pass": finite and ratio <= 1.0}
