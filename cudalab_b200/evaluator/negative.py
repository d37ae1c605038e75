"""Negative-case runner: the contract of the reference's generic negative
runner (cudalab/evaluator/negative.py:113-155), implemented here.

Contract
  * An illegal input must be refused on the host, before any device work.
    Whatever exception the call raises counts as a refusal.
  * Where a case names a message fragment, the refusal's first line must
    contain it (the suites pin the reference's validation texts this way).
  * A legal input ("pass" cases) must run without raising.
  * After every non-skipped case a control call proves the CUDA context is
    still usable, so a refusal that corrupted the device fails its case.

Each case yields one JSON-ready record:
  outcome          "refused" | "ran" | "skipped"
  error            exception class name of a refusal
  first_line       first line of its message (300 characters at most)
  wanted_fragment  the fragment the case names, or None
  fragment_found   None when nothing was asked or nothing raised, else bool
  context_healthy  result of the control call (None when skipped)
  pass             the verdict (absent for skipped cases)
`summarize_cases` folds the records into counts plus `all_pass`.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

EXPECTATIONS = ("reject", "pass", "skip")


def _attempt(call: Callable[[], None]) -> tuple[Optional[str], Optional[str]]:
    """(exception class, first message line) of a refusal, (None, None) when
    the call returns."""
    try:
        call()
    except Exception as exc:  # noqa: BLE001 - the contract counts every exception
        lines = str(exc).splitlines()
        return type(exc).__name__, (lines[0][:300] if lines else "")
    return None, None


def run_case(variant: str, description: str, call: Callable[[], None], expected: str,
             expect_msg_contains: Optional[str], control_ok: Callable[[], bool]) -> dict:
    """Run one case and return its record.  `expected` is one of
    "reject" | "pass" | "skip"; `control_ok` runs a legal call and returns
    whether the context is healthy (not called for skipped cases)."""
    if expected not in EXPECTATIONS:
        raise ValueError(f"expected must be one of {EXPECTATIONS}, got {expected!r}")
    torch.cuda.synchronize()
    error, line = _attempt(call)
    refused = error is not None
    found = None
    if expect_msg_contains and refused:
        found = expect_msg_contains in line
    rec = {"variant": variant, "description": description, "expected": expected,
           "error": error, "first_line": line, "wanted_fragment": expect_msg_contains,
           "fragment_found": found}
    if expected == "skip":
        rec.update(outcome="skipped", context_healthy=None)
        return rec
    healthy = bool(control_ok())
    rec.update(outcome="refused" if refused else "ran", context_healthy=healthy)
    if expected == "reject":
        rec["pass"] = refused and healthy and found is not False
    else:
        rec["pass"] = (not refused) and healthy
    return rec


def summarize_cases(results: list[dict]) -> dict:
    """Counts per expectation and the overall verdict; skipped cases never
    fail a suite."""
    judged = [r for r in results if r["expected"] != "skip"]
    passed = [r for r in judged if r.get("pass")]

    def count(rs, exp):
        return sum(1 for r in rs if r["expected"] == exp)

    return {
        "n_total": len(results),
        "n_judged": len(judged),
        "n_passed": len(passed),
        "n_failed": len(judged) - len(passed),
        "n_skipped": len(results) - len(judged),
        "refusals_expected": count(judged, "reject"),
        "refusals_ok": count(passed, "reject"),
        "legal_expected": count(judged, "pass"),
        "legal_ok": count(passed, "pass"),
        "all_pass": len(passed) == len(judged),
    }
