"""CPU oracle of RMSNorm and of the fused RMSNorm -> INT4 GEMV (test
infrastructure only: imported by tests/, never by the package).

RMSNorm restates cudalab/reference.py:19-44 (rmsnorm_ref): with x32 = x in
fp32, v = mean(x32^2) accumulated in fp32, y = fp16((x32 * rsqrt(v + eps)) *
w32).  The reduction order of the mean is not part of the contract (torch's
CPU reduction and the GPU's block reduction differ in the last bits of v), so
the oracle computes the normalisation in fp64 and an output is accepted when
every element is within one fp16 ulp of the correctly rounded fp64 value.

The fused operator is y[m] = W x_norm[m] with x_norm = RMSNorm(x[m], g): the
reference's fixed arithmetic bound of the INT4 GEMV (cudalab/
int4gemv_correctness.py:175-209, restated in int4gemv_oracle.arith_ratio)
applied to the fp64 exact product with x_norm, widened by one fp16 ulp of
every normalised activation: |y - exact| <= TOL_K (3 K u S + ulp16(y) / 2 +
ulp16(exact) / 2) + sum_k |q s|_k ulp16(x_norm_k).

Pinned by tests/golden/rmsnorm_golden.npz (made by the reference's own
make_inputs / rmsnorm_ref / quantiser; tests/test_golden_cpu.py).
"""
from __future__ import annotations

import numpy as np

from . import int4gemv_oracle as o4

EPS = 1e-5


def rmsnorm_exact(x16: np.ndarray, w16: np.ndarray, eps: float = EPS) -> np.ndarray:
    """fp64 RMSNorm of fp16 rows x [M, H] with weight w [H] (not rounded)."""
    x = np.asarray(x16, np.float16).astype(np.float64)
    w = np.asarray(w16, np.float16).astype(np.float64)
    v = np.mean(x * x, axis=-1, keepdims=True)
    return x / np.sqrt(v + eps) * w


def ulp16(v: np.ndarray) -> np.ndarray:
    return o4.ulp16(v)


def rmsnorm_check(y16: np.ndarray, x16: np.ndarray, w16: np.ndarray, eps: float = EPS) -> dict:
    """Every element within one fp16 ulp of the correctly rounded fp64 value."""
    ex = rmsnorm_exact(x16, w16, eps)
    y = np.asarray(y16, np.float16).astype(np.float64)
    rounded = ex.astype(np.float16).astype(np.float64)
    err = np.abs(y - rounded) / ulp16(rounded)
    finite = bool(np.isfinite(y).all())
    worst = float(err.max()) if err.size else 0.0
    return {"max_ulp": worst, "finite": finite, "pass": finite and worst <= 1.0}


def fused_check(y16: np.ndarray, Wp: np.ndarray, scale16: np.ndarray, x16: np.ndarray,
                g16: np.ndarray, eps: float = EPS) -> dict:
    """Rows y16 [M, n] of the fused operator against the widened bound, for
    the weight rows Wp [n, K/2] / scale16 [n, K/128] and activations x16 [M, K]."""
    xn = rmsnorm_exact(x16, g16, eps).astype(np.float16)
    a = o4.unpack_w(Wp).astype(np.float64) * np.repeat(scale16.astype(np.float64), o4.GROUP,
                                                        axis=1)
    K = 2 * Wp.shape[1]
    worst, finite = 0.0, bool(np.isfinite(np.asarray(y16, np.float32)).all())
    for m in range(xn.shape[0]):
        xd = xn[m].astype(np.float64)
        exact = a @ xd
        S = np.abs(a) @ np.abs(xd)
        slack = np.abs(a) @ ulp16(xd)
        yd = np.asarray(y16[m], np.float16).astype(np.float64)
        tol = o4.TOL_K * (o4.ROUNDINGS * K * o4.U * S + 0.5 * ulp16(yd) + 0.5 * ulp16(exact)) \
            + slack
        with np.errstate(invalid="ignore", divide="ignore"):
            r = np.abs(yd - exact) / tol
        r = np.where(np.isfinite(r), r, 0.0)
        worst = max(worst, float(r.max()) if r.size else 0.0)
    return {"ratio": worst, "finite": finite, "pass": finite and worst <= 1.0}
