"""Dense GEMV correctness suite (the reference's cudalab/gemv_correctness.py).

Gate per case (fixed for every variant, never relaxed;
cudalab/gemv_correctness.py:59-73,163-191 of the reference):
  * exact = fp64 GEMV of the stored values (a_k = W[n,k] * x[k], exact);
  * tol_n = TOL_K * (2 K 2^-24 S_n + ulp(y_n)/2 + ulp(exact_n)/2) on the grid
    of the element type, S_n = sum_k |a_k| -- the bound of any fp32
    evaluation order in which each term sees at most 2 roundings;
  * pass iff max_n |y_n - exact_n| / tol_n <= 1 and y and the reference
    result are finite.
The elementwise comparison against gemv_ref (fp16: fp16(mv(W.float(),
x.float())); fp32: mv(W, x)) with the shared tolerances is reported only.

Matrix: float16 and float32 x the five benchmark shapes plus five edge shapes
x five input modes, W seed 0 / x seed 1 (independent streams), large = 10
(cudalab/gemv_correctness.py:111-121,241-261): 100 checks per variant.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass

import torch

from .evaluator.correctness import TOLERANCES, compute_metrics, summarize_results
from .operators.gemv import BENCH_MATRIX_GEMV, gemv_ref, make_w, make_x

DTYPES = ("float16", "float32")
EDGE_SHAPES = [(1, 1), (1, 4096), (4096, 1), (16, 13), (8, 7)]
SHAPES = list(BENCH_MATRIX_GEMV) + EDGE_SHAPES
INPUT_MODES = ("normal", "zeros", "tiny", "large", "mixed_sign")
LARGE_SCALE = 10.0
SEED = 0
TOL_K = 2.0
PER_TERM_ROUNDINGS = 2.0
_U = 2.0 ** -24


def ulp(v: torch.Tensor, dtype_name: str) -> torch.Tensor:
    """Spacing of the element type's grid at v (fp16: 2^-24 in the subnormal
    range; fp32: distance to the next float up)."""
    if dtype_name == "float32":
        vf = v.float()
        return (torch.nextafter(vf, torch.full_like(vf, float("inf"))) - vf).double()
    a = v.to(torch.float16).to(torch.float64).abs()
    _, e = torch.frexp(a.clamp_min(2.0 ** -14))   # a = m * 2^e, m in [0.5, 1)
    u = torch.ldexp(torch.ones_like(a), (e - 11).to(torch.int32))
    return torch.where(a >= 2.0 ** -14, u, torch.full_like(a, 2.0 ** -24))


def exact_and_S(W: torch.Tensor, x: torch.Tensor):
    wd, xd = W.cpu().double(), x.cpu().double()
    return wd @ xd, wd.abs() @ xd.abs()


def arith_ratio(y: torch.Tensor, W: torch.Tensor, x: torch.Tensor, dtype_name: str,
                exact=None, S=None):
    """(max ratio, max tol, max S); non-finite entries count 0 here (the
    finiteness gate catches them)."""
    if W.numel() == 0:
        return 0.0, 0.0, 0.0
    K = W.shape[1]
    if exact is None or S is None:
        exact, S = exact_and_S(W, x)
    yd = y.cpu().double()
    tol = TOL_K * (PER_TERM_ROUNDINGS * K * _U * S + 0.5 * ulp(yd, dtype_name)
                   + 0.5 * ulp(exact, dtype_name))
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
    atol: float
    rtol: float
    note: str = ""


class _Case:
    """Inputs (host) plus reference values of one (dtype, shape, mode) case."""

    def __init__(self, dtype_name: str, N: int, K: int, mode: str):
        self.dtype_name, self.N, self.K, self.mode = dtype_name, N, K, mode
        dt = getattr(torch, dtype_name)
        self.W = make_w(N, K, dtype=dt, seed=SEED, mode=mode, large=LARGE_SCALE)
        self.x = make_x(K, dtype=dt, seed=SEED + 1, mode=mode, large=LARGE_SCALE)
        self.ref = gemv_ref(self.W, self.x)
        self.exact, self.S = exact_and_S(self.W, self.x)


_CACHE: dict = {}


def get_case(dtype_name: str, N: int, K: int, mode: str) -> _Case:
    key = (dtype_name, N, K, mode)
    if key not in _CACHE:
        _CACHE[key] = _Case(dtype_name, N, K, mode)
    return _CACHE[key]


def check_case(variant: str, ext, case: _Case, device: str = "cuda") -> CheckResult:
    y = ext.forward(variant, case.W.to(device), case.x.to(device)).cpu()
    ratio, tol_max, S_max = arith_ratio(y, case.W, case.x, case.dtype_name,
                                        exact=case.exact, S=case.S)
    ref_nan = bool(torch.isnan(case.ref).any())
    ref_inf = bool(torch.isinf(case.ref).any())
    m = compute_metrics(y, case.ref, case.dtype_name)
    return CheckResult(
        variant=variant, shape=[case.N, case.K], dtype=case.dtype_name, seed=SEED,
        mode=case.mode,
        passed=(ratio <= 1.0 and not m["has_nan"] and not m["has_inf"]
                and not ref_nan and not ref_inf),
        arith_max_ratio=round(ratio, 12), has_nan=m["has_nan"], has_inf=m["has_inf"],
        ref_has_nan=ref_nan, ref_has_inf=ref_inf, max_abs_error=m["max_abs_error"],
        max_rel_error=m["max_rel_error"], ok_close=m["ok_close"],
        arith_tol_max=round(tol_max, 12), S_max=round(S_max, 12),
        atol=m["atol"], rtol=m["rtol"],
        note="" if not (ref_nan or ref_inf) else "reference not finite: suite construction error")


def run_suite(variant: str, ext, dtypes=DTYPES, shapes=SHAPES,
              modes=INPUT_MODES) -> list[CheckResult]:
    """2 dtypes x 10 shapes x 5 modes for one variant (deterministic)."""
    return [check_case(variant, ext, get_case(dt, N, K, mode))
            for dt in dtypes for (N, K) in shapes for mode in modes]


def _jsonable(r: CheckResult) -> dict:
    d = asdict(r)
    d["pass"] = d.pop("passed")
    return d


def summarize(results: list[CheckResult]) -> dict:
    s = summarize_results([_jsonable(r) for r in results])
    s["max_arith_max_ratio"] = max((r.arith_max_ratio for r in results), default=0.0)
    s["ok_close_vs_ref_all"] = all(r.ok_close for r in results)
    s["tolerances_reported"] = TOLERANCES
    s["tol_k"] = TOL_K
    return s
