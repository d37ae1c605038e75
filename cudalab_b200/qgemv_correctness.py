"""INT8 GEMV kernel-correctness suite (the reference's layer A,
cudalab/qgemv_correctness.py): same fixed fp64 arithmetic gate as the INT4
suite with a_k = q * s * x, s the stored fp32 row scale
(cudalab/qgemv_correctness.py:152-168).  Matrix: five benchmark shapes plus
edge shapes (1,1) (1,4096) (4096,1) (16,13) (8,7) x five modes, W seed 0,
x seed 1 (cudalab/qgemv_correctness.py:93-100).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Optional

import torch

from .evaluator.correctness import TOLERANCES, compute_metrics, summarize_results
from .int4gemv_correctness import PER_TERM_ROUNDINGS, TOL_K, ulp16
from .operators.qgemv import BENCH_MATRIX_QGEMV, make_w_q, make_x_q
from .qgemv_quantize import dequantize_w, fidelity_metrics

DTYPES = ("float16",)
EDGE_SHAPES = [(1, 1), (1, 4096), (4096, 1), (16, 13), (8, 7)]
SHAPES = list(BENCH_MATRIX_QGEMV) + EDGE_SHAPES
INPUT_MODES = ("normal", "zeros", "tiny", "large", "mixed_sign")
LARGE_SCALE = 10.0
SEED = 0
_U = 2.0 ** -24
_ROW_CHUNK = 1024


def exact_and_S(W_q: torch.Tensor, scale: torch.Tensor, x: torch.Tensor):
    Wq, s, xd = W_q.cpu(), scale.cpu(), x.cpu().double()
    N = Wq.shape[0]
    ex = torch.empty(N, dtype=torch.float64)
    S = torch.empty(N, dtype=torch.float64)
    for r0 in range(0, N, _ROW_CHUNK):
        r1 = min(N, r0 + _ROW_CHUNK)
        a = Wq[r0:r1].double() * s[r0:r1].double().unsqueeze(1)
        ex[r0:r1] = a @ xd
        S[r0:r1] = a.abs() @ xd.abs()
    return ex, S


def arith_ratio(y, W_q, scale, x, dtype_name: str = "float16", exact=None, S=None):
    if W_q.numel() == 0:
        return 0.0, 0.0, 0.0
    K = W_q.shape[1]
    if exact is None or S is None:
        exact, S = exact_and_S(W_q, scale, x)
    yd = y.cpu().double()
    tol = TOL_K * (PER_TERM_ROUNDINGS * K * _U * S + 0.5 * ulp16(yd) + 0.5 * ulp16(exact))
    diff = (yd - exact).abs()
    ratio = torch.where(diff.isfinite() & tol.isfinite(), diff / tol, torch.zeros_like(diff))
    return float(ratio.max()), float(tol.max()), float(S.max())


@dataclass
class CheckResult:
    variant: str
    shape: list
    dtype: str
    seed: int
    mode: str
    passed: bool
    arith_max_ratio: float
    has_nan: bool
    has_inf: bool
    ref_has_nan: bool
    ref_has_inf: bool
    max_abs_error: float
    max_rel_error: float
    ok_close: bool
    arith_tol_max: float
    S_max: float
    fid_max_abs: Optional[float]
    fid_max_rel: Optional[float]
    fid_rmse: Optional[float]
    fid_cosine: Optional[float]
    atol: float
    rtol: float
    note: str = ""


class _Case:
    def __init__(self, N: int, K: int, mode: str):
        self.N, self.K, self.mode = N, K, mode
        self.W_q, self.scale, self.W_fp16 = make_w_q(N, K, seed=SEED, mode=mode,
                                                     large=LARGE_SCALE, device="cpu")
        self.x = make_x_q(K, seed=SEED + 1, mode=mode, large=LARGE_SCALE, device="cpu")
        self.ref = torch.mv(dequantize_w(self.W_q, self.scale), self.x.float()).to(torch.float16)
        self.exact, self.S = exact_and_S(self.W_q, self.scale, self.x)
        self.fid = fidelity_metrics(self.W_fp16, self.x, self.W_q, self.scale)


_CACHE: dict = {}


def get_case(N: int, K: int, mode: str) -> _Case:
    key = (N, K, mode)
    if key not in _CACHE:
        _CACHE[key] = _Case(N, K, mode)
    return _CACHE[key]


def check_case(variant: str, ext, case: _Case, device: str = "cuda") -> CheckResult:
    y = ext.forward(variant, case.W_q.to(device), case.scale.to(device),
                    case.x.to(device)).cpu()
    ratio, tol_max, S_max = arith_ratio(y, case.W_q, case.scale, case.x,
                                        exact=case.exact, S=case.S)
    ref_nan = bool(torch.isnan(case.ref).any())
    ref_inf = bool(torch.isinf(case.ref).any())
    m = compute_metrics(y, case.ref, "float16")
    fid = case.fid
    return CheckResult(
        variant=variant, shape=[case.N, case.K], dtype="float16", seed=SEED, mode=case.mode,
        passed=(ratio <= 1.0 and not m["has_nan"] and not m["has_inf"]
                and not ref_nan and not ref_inf),
        arith_max_ratio=round(ratio, 12), has_nan=m["has_nan"], has_inf=m["has_inf"],
        ref_has_nan=ref_nan, ref_has_inf=ref_inf, max_abs_error=m["max_abs_error"],
        max_rel_error=m["max_rel_error"], ok_close=m["ok_close"],
        arith_tol_max=round(tol_max, 12), S_max=round(S_max, 12),
        fid_max_abs=round(fid["max_abs"], 12), fid_max_rel=round(fid["max_rel"], 12),
        fid_rmse=round(fid["rmse"], 12),
        fid_cosine=(round(fid["cosine"], 9) if fid["cosine"] is not None else None),
        atol=m["atol"], rtol=m["rtol"],
        note="" if not (ref_nan or ref_inf) else "reference not finite: suite construction error")


def run_suite(variant: str, ext, shapes=SHAPES, modes=INPUT_MODES) -> list[CheckResult]:
    return [check_case(variant, ext, get_case(N, K, mode)) for (N, K) in shapes for mode in modes]


def _jsonable(r: CheckResult) -> dict:
    d = asdict(r)
    d["pass"] = d.pop("passed")
    return d


def summarize(results: list[CheckResult]) -> dict:
    s = summarize_results([_jsonable(r) for r in results])
    s["max_arith_max_ratio"] = max((r.arith_max_ratio for r in results), default=0.0)
    s["ok_close_vs_ref_all"] = all(r.ok_close for r in results)
    s["tolerances_reported"] = TOLERANCES["float16"]
    s["tol_k"] = TOL_K
    return s
