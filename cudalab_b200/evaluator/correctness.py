"""Fixed report-only tolerances and elementwise metrics
(role of cudalab/evaluator/correctness.py:27-90).

The pass/fail gate of the GEMV suites is the fixed arithmetic bound of the
suite modules; the elementwise allclose below is reported, never gating.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

TOLERANCES = {
    "float16": {"atol": 2e-3, "rtol": 5e-3},
    "float32": {"atol": 1e-5, "rtol": 1e-4},
}
REL_EPS_GUARD = 1e-3


def compute_metrics(y: torch.Tensor, ref: torch.Tensor, dtype_name: str,
                    rel_eps_guard: float = REL_EPS_GUARD) -> dict:
    tol = TOLERANCES[dtype_name]
    yf, rf = y.float(), ref.float()
    diff = (yf - rf).abs()
    n = y.numel()
    return {
        "max_abs_error": round(float(diff.max()) if n else 0.0, 12),
        "max_rel_error": round(float((diff / rf.abs().clamp_min(rel_eps_guard)).max())
                               if n else 0.0, 12),
        "has_nan": bool(torch.isnan(y).any()),
        "has_inf": bool(torch.isinf(y).any()),
        "ok_close": bool(torch.allclose(yf, rf, atol=tol["atol"], rtol=tol["rtol"])),
        "atol": tol["atol"],
        "rtol": tol["rtol"],
    }


def summarize_results(results: list[dict]) -> dict:
    failed = [r for r in results if not r["pass"]]
    return {
        "n_total": len(results),
        "n_pass": len(results) - len(failed),
        "n_fail": len(failed),
        "all_pass": not failed,
        "max_abs_error": max((r["max_abs_error"] for r in results), default=0.0),
        "max_rel_error": max((r["max_rel_error"] for r in results), default=0.0),
        "failed": failed[:20],
    }


def save_suite(path: Path, doc: dict) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(doc, indent=2, ensure_ascii=False))
    return path
