"""INT4 GEMV kernel-correctness suite (the reference's layer A,
cudalab/int4gemv_correctness.py).

Gate per case (fixed for every variant, never relaxed):
  * exact = fp64 GEMV of the stored values, a_k = q * s16 * x (exact products);
  * tol_n = TOL_K * (3 K 2^-24 S_n + ulp16(y_n)/2 + ulp16(exact_n)/2),
    S_n = sum_k |a_k|  -- the bound of any fp32 evaluation order in which each
    term sees at most 3 roundings (cudalab/int4gemv_correctness.py:175-209);
  * pass iff max_n |y_n - exact_n| / tol_n <= 1 and y, ref are finite.
The elementwise comparison against ref = fp16(mv(dequant(W), x)) with the fp16
tolerances is reported, not gating.

Matrix: the five benchmark shapes plus five edge shapes x five input modes,
W seed 0, x seed 1 (cudalab/int4gemv_correctness.py:117-121,263-284).
Reference values are computed on the host from the stored fp16 scale.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Optional

import torch

from .evaluator.correctness import TOLERANCES, compute_metrics, summarize_results
from .int4gemv_quantize import GROUP_SIZE, dequantize_w, fidelity_metrics, unpack_w
from .operators.int4gemv import BENCH_MATRIX_INT4GEMV, make_w4, make_x4

DTYPES = ("float16",)
EDGE_SHAPES = [(1, 128), (1, 4096), (3, 128), (16, 256), (8, 128)]
SHAPES = list(BENCH_MATRIX_INT4GEMV) + EDGE_SHAPES
INPUT_MODES = ("normal", "zeros", "tiny", "large", "mixed_sign")
LARGE_SCALE = 10.0
SEED = 0
TOL_K = 2.0
PER_TERM_ROUNDINGS = 3.0
_U = 2.0 ** -24
_ROW_CHUNK = 1024


def ulp16(v: torch.Tensor) -> torch.Tensor:
    """Spacing of the binary16 grid at fp16(v) (2^-24 in the subnormal range)."""
    a = v.to(torch.float16).to(torch.float64).abs()
    _, e = torch.frexp(a.clamp_min(2.0 ** -14))   # a = m * 2^e, m in [0.5, 1)
    u = torch.ldexp(torch.ones_like(a), (e - 11).to(torch.int32))
    return torch.where(a >= 2.0 ** -14, u, torch.full_like(a, 2.0 ** -24))


def exact_and_S(W_packed: torch.Tensor, scale: torch.Tensor, x: torch.Tensor):
    """fp64 exact GEMV and S_n = sum_k |q s x| (host, row-chunked)."""
    Wp, s16, xd = W_packed.cpu(), scale.cpu(), x.cpu().double()
    N = Wp.shape[0]
    ex = torch.empty(N, dtype=torch.float64)
    S = torch.empty(N, dtype=torch.float64)
    for r0 in range(0, N, _ROW_CHUNK):
        r1 = min(N, r0 + _ROW_CHUNK)
        a = unpack_w(Wp[r0:r1]).double() * \
            s16[r0:r1].double().repeat_interleave(GROUP_SIZE, dim=1)
        ex[r0:r1] = a @ xd
        S[r0:r1] = a.abs() @ xd.abs()
    return ex, S


def arith_ratio(y: torch.Tensor, W_packed: torch.Tensor, scale: torch.Tensor,
                x: torch.Tensor, dtype_name: str = "float16", exact=None, S=None):
    """(max ratio, max tol, max S) of the fixed bound; non-finite entries count
    0 here (the finiteness gate catches them)."""
    if W_packed.numel() == 0:
        return 0.0, 0.0, 0.0
    K = 2 * W_packed.shape[1]
    if exact is None or S is None:
        exact, S = exact_and_S(W_packed, scale, x)
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
    fid_rmse: Optional[float]
    fid_cosine: Optional[float]
    atol: float
    rtol: float
    note: str = ""


class _Case:
    """Inputs plus host-side reference values of one (shape, mode) case."""

    def __init__(self, N: int, K: int, mode: str):
        self.N, self.K, self.mode = N, K, mode
        self.W_packed, self.scale, self.W_fp16 = make_w4(N, K, seed=SEED, mode=mode,
                                                         large=LARGE_SCALE, device="cpu")
        self.x = make_x4(K, seed=SEED + 1, mode=mode, large=LARGE_SCALE, device="cpu")
        self.ref = torch.mv(dequantize_w(self.W_packed, self.scale),
                            self.x.float()).to(torch.float16)
        self.exact, self.S = exact_and_S(self.W_packed, self.scale, self.x)
        self.fid = fidelity_metrics(self.W_fp16, self.x, self.W_packed, self.scale)


_CACHE: dict = {}


def get_case(N: int, K: int, mode: str) -> _Case:
    key = (N, K, mode)
    if key not in _CACHE:
        _CACHE[key] = _Case(N, K, mode)
    return _CACHE[key]


def check_case(variant: str, ext, case: _Case, device: str = "cuda") -> CheckResult:
    y = ext.forward(variant, case.W_packed.to(device), case.scale.to(device),
                    case.x.to(device)).cpu()
    ratio, tol_max, S_max = arith_ratio(y, case.W_packed, case.scale, case.x,
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
        fid_max_abs=round(fid["max_abs"], 12), fid_rmse=round(fid["rmse"], 12),
        fid_cosine=(round(fid["cosine"], 9) if fid["cosine"] is not None else None),
        atol=m["atol"], rtol=m["rtol"],
        note="" if not (ref_nan or ref_inf) else "reference not finite: suite construction error")


def run_suite(variant: str, ext, shapes=SHAPES, modes=INPUT_MODES) -> list[CheckResult]:
    """All 10 shapes x 5 modes for one variant (deterministic)."""
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
