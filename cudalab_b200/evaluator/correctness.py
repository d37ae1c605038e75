"""Report-only elementwise comparison and suite summaries.

The reference reports an elementwise allclose beside its gate but never
decides with it (cudalab/evaluator/correctness.py:27-30): the pass/fail
decision of every GEMV suite here is the fixed arithmetic bound of the suite
modules.  This module supplies the reported figures and the summary of a list
of check records.

`TOLERANCES` holds the reference's fixed report tolerances per dtype (fp16:
atol 2e-3, rtol 5e-3; fp32: atol 1e-5, rtol 1e-4) and `REL_EPS_GUARD` the
floor of the relative-error denominator; both are constants of the interface,
so reported numbers are comparable with the reference's records.
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
_DIGITS = 12  # small errors (1e-9 and below) stay visible in the records


def compute_metrics(y: torch.Tensor, ref: torch.Tensor, dtype_name: str,
                    rel_eps_guard: float = REL_EPS_GUARD) -> dict:
    """Elementwise figures of y against ref, both compared in fp32:
    largest absolute and relative error (relative to max(|ref|, guard)),
    non-finite flags of y, and the report-only allclose at the dtype's
    tolerances (echoed as atol / rtol)."""
    atol, rtol = TOLERANCES[dtype_name]["atol"], TOLERANCES[dtype_name]["rtol"]
    a, b = y.detach().float().flatten(), ref.detach().float().flatten()
    if a.numel() == 0:
        worst_abs = worst_rel = 0.0
        close = True
    else:
        err = torch.abs(a - b)
        worst_abs = err.max().item()
        worst_rel = (err / torch.clamp(torch.abs(b), min=rel_eps_guard)).max().item()
        close = bool((err <= atol + rtol * torch.abs(b)).all().item())
    finite_mask = torch.isfinite(a)
    return {
        "max_abs_error": round(float(worst_abs), _DIGITS),
        "max_rel_error": round(float(worst_rel), _DIGITS),
        "has_nan": bool(torch.isnan(a).any().item()),
        "has_inf": bool((~finite_mask & ~torch.isnan(a)).any().item()),
        "ok_close": close,
        "atol": atol,
        "rtol": rtol,
    }


def summarize_results(results: list[dict]) -> dict:
    """Counts, verdict and worst errors of a suite's records (each has at
    least "pass", "max_abs_error", "max_rel_error"); the first 20 failing
    records are kept whole."""
    fails = []
    worst_abs = worst_rel = 0.0
    for r in results:
        worst_abs = max(worst_abs, r["max_abs_error"])
        worst_rel = max(worst_rel, r["max_rel_error"])
        if not r["pass"]:
            fails.append(r)
    return {
        "n_total": len(results),
        "n_pass": len(results) - len(fails),
        "n_fail": len(fails),
        "all_pass": len(fails) == 0,
        "max_abs_error": worst_abs,
        "max_rel_error": worst_rel,
        "failed": fails[:20],
    }


def save_suite(path: Path, doc: dict) -> Path:
    """Write a suite document as UTF-8 JSON (the reference's messages are
    Chinese, kept readable), creating the directory."""
    out = Path(path)
    out.parent.mkdir(parents=True, exist_ok=True)
    with out.open("w", encoding="utf-8") as fh:
        json.dump(doc, fh, indent=2, ensure_ascii=False)
    return out
