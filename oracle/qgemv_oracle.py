"""TEST INFRASTRUCTURE ONLY (checker, never the product path).

numpy restatement of the reference's INT8 weight-only algorithm:
  quantize_w     cudalab/qgemv_quantize.py:33-64 (fp32 row scale, stored fp32)
  dequantize_w   cudalab/qgemv_quantize.py:67-70
  layer-A ref    cudalab/qgemv_correctness.py:157-158
  arith gate     cudalab/qgemv_correctness.py:118-150
Parity pinned by tests/golden/qgemv_golden.npz (reference outputs).
"""
from __future__ import annotations

import numpy as np

from .int4gemv_oracle import ROUNDINGS, TOL_K, U, ulp16

QMAX = 127


def quantize_w(W: np.ndarray):
    assert W.dtype == np.float16 and W.ndim == 2
    Wf = W.astype(np.float32)
    s = (np.abs(Wf).max(axis=1) / np.float32(QMAX)).astype(np.float32)
    zero = s == 0
    den = np.where(zero, np.float32(1.0), s).astype(np.float32)[:, None]
    q = np.clip(np.rint(Wf / den), -QMAX, QMAX)
    q = np.where(zero[:, None], 0.0, q)
    return q.astype(np.int8), s


def dequantize_w(Wq: np.ndarray, s: np.ndarray) -> np.ndarray:
    return Wq.astype(np.float32) * s.astype(np.float32)[:, None]


def gemv_ref(Wq: np.ndarray, s: np.ndarray, x16: np.ndarray) -> np.ndarray:
    return (dequantize_w(Wq, s) @ x16.astype(np.float32)).astype(np.float16)


def exact_and_S(Wq: np.ndarray, s: np.ndarray, x16: np.ndarray, row_chunk: int = 2048):
    N = Wq.shape[0]
    xd = x16.astype(np.float64)
    ex = np.empty(N, np.float64)
    S = np.empty(N, np.float64)
    for r0 in range(0, N, row_chunk):
        r1 = min(N, r0 + row_chunk)
        a = Wq[r0:r1].astype(np.float64) * s[r0:r1].astype(np.float64)[:, None]
        ex[r0:r1] = a @ xd
        S[r0:r1] = np.abs(a) @ np.abs(xd)
    return ex, S


def arith_ratio(y16: np.ndarray, K: int, exact: np.ndarray, S: np.ndarray) -> float:
    yd = y16.astype(np.float64)
    tol = TOL_K * (ROUNDINGS * K * U * S + 0.5 * ulp16(yd) + 0.5 * ulp16(exact))
    with np.errstate(invalid="ignore", divide="ignore"):
        r = np.abs(yd - exact) / tol
    r = np.where(np.isfinite(r), r, 0.0)
    return float(r.max()) if r.size else 0.0


def check(y16: np.ndarray, Wq: np.ndarray, s: np.ndarray, x16: np.ndarray) -> dict:
    ex, S = exact_and_S(Wq, s, x16)
    ratio = arith_ratio(y16, Wq.shape[1], ex, S)
    finite = bool(np.isfinite(y16.astype(np.float32)).all())
    return {"arith_max_ratio": ratio, "finite": finite, "pass": finite and ratio <= 1.0}
