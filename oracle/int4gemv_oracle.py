"""TEST INFRASTRUCTURE ONLY (checker, never the product path).

numpy restatement of the reference's W4A16 algorithm:
  quantize_w     cudalab/int4gemv_quantize.py:61-89
  pack_q         cudalab/int4gemv_quantize.py:92-114
  unpack_w       cudalab/int4gemv_quantize.py:117-134
  dequantize_w   cudalab/int4gemv_quantize.py:137-149
  layer-A ref    cudalab/int4gemv_correctness.py:220-221 (fp32 mv -> fp16)
  arith gate     cudalab/int4gemv_correctness.py:124-125,175-209
Parity pinned by tests/golden/int4gemv_golden.npz (reference outputs).
"""
from __future__ import annotations

import numpy as np

GROUP = 128
QMAX = 7
TOL_K = 2.0
ROUNDINGS = 3.0
U = 2.0 ** -24


def quantize_w(W: np.ndarray):
    """fp16 [N, K] -> (uint8 [N, K/2], fp16 [N, K/128]); fp32 arithmetic,
    round-half-even (np.rint), clamp to [-7, 7], zero group -> q = 0."""
    assert W.dtype == np.float16 and W.ndim == 2 and W.shape[1] % GROUP == 0
    N, K = W.shape
    g = W.astype(np.float32).reshape(N, K // GROUP, GROUP)
    s32 = (np.abs(g).max(axis=2) / np.float32(QMAX)).astype(np.float32)
    zero = s32 == 0
    den = np.where(zero, np.float32(1.0), s32).astype(np.float32)[:, :, None]
    q = np.clip(np.rint(g / den), -QMAX, QMAX)
    q = np.where(zero[:, :, None], 0.0, q).astype(np.int32).reshape(N, K)
    return pack_q(q), s32.astype(np.float16)


def pack_q(q: np.ndarray) -> np.ndarray:
    N, K = q.shape
    assert K % 2 == 0 and q.min(initial=0) >= -8 and q.max(initial=0) <= 7
    p = (q.astype(np.int32) & 0xF).reshape(N, K // 2, 2)
    return (p[..., 0] | (p[..., 1] << 4)).astype(np.uint8)


def unpack_w(Wp: np.ndarray) -> np.ndarray:
    b = Wp.astype(np.int32)
    lo, hi = b & 0xF, (b >> 4) & 0xF
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    return np.stack([lo, hi], axis=-1).reshape(Wp.shape[0], 2 * Wp.shape[1])


def dequantize_w(Wp: np.ndarray, scale16: np.ndarray) -> np.ndarray:
    q = unpack_w(Wp).astype(np.float32)
    return q * np.repeat(scale16.astype(np.float32), GROUP, axis=1)


def gemv_ref(Wp: np.ndarray, scale16: np.ndarray, x16: np.ndarray) -> np.ndarray:
    """Layer-A reference: fp32 dequantised GEMV, cast to fp16."""
    return (dequantize_w(Wp, scale16) @ x16.astype(np.float32)).astype(np.float16)


def exact_and_S(Wp: np.ndarray, scale16: np.ndarray, x16: np.ndarray, row_chunk: int = 2048):
    """fp64 exact GEMV of the stored values and S_n = sum_k |q s x|."""
    N = Wp.shape[0]
    xd = x16.astype(np.float64)
    ex = np.empty(N, np.float64)
    S = np.empty(N, np.float64)
    for r0 in range(0, N, row_chunk):
        r1 = min(N, r0 + row_chunk)
        a = unpack_w(Wp[r0:r1]).astype(np.float64) * \
            np.repeat(scale16[r0:r1].astype(np.float64), GROUP, axis=1)
        ex[r0:r1] = a @ xd
        S[r0:r1] = np.abs(a) @ np.abs(xd)
    return ex, S


def ulp16(v: np.ndarray) -> np.ndarray:
    """binary16 grid spacing at fp16(v); 2^-24 below the normal range."""
    a = np.abs(np.asarray(v, np.float64).astype(np.float16).astype(np.float64))
    with np.errstate(divide="ignore", invalid="ignore"):
        _, e = np.frexp(np.maximum(a, 2.0 ** -14))
    u = np.ldexp(1.0, e - 11)
    return np.where(a >= 2.0 ** -14, u, 2.0 ** -24)


def arith_ratio(y16: np.ndarray, K: int, exact: np.ndarray, S: np.ndarray) -> float:
    """max_n |y - exact| / (TOL_K (3 K 2^-24 S + ulp16(y)/2 + ulp16(exact)/2))."""
    yd = y16.astype(np.float64)
    tol = TOL_K * (ROUNDINGS * K * U * S + 0.5 * ulp16(yd) + 0.5 * ulp16(exact))
    with np.errstate(invalid="ignore", divide="ignore"):
        r = np.abs(yd - exact) / tol
    r = np.where(np.isfinite(r), r, 0.0)
    return float(r.max()) if r.size else 0.0


def check(y16: np.ndarray, Wp: np.ndarray, scale16: np.ndarray, x16: np.ndarray) -> dict:
    """Full layer-A verdict of an output against the oracle."""
    ex, S = exact_and_S(Wp, scale16, x16)
    ratio = arith_ratio(y16, 2 * Wp.shape[1], ex, S)
    finite = bool(np.isfinite(y16.astype(np.float32)).all())
    return {"arith_max_ratio": ratio, "finite": finite, "pass": finite and ratio <= 1.0}
