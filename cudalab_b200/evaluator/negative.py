"""Negative-case runner (role of cudalab/evaluator/negative.py:113-155).

An illegal input must raise before any kernel launch; any exception counts as
a rejection, and when `expect_msg_contains` is given the first line of the
message must contain it.  After every case a control forward checks that the
CUDA context is still healthy.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch


def run_case(variant: str, description: str, call: Callable[[], None], expected: str,
             expect_msg_contains: Optional[str], control_ok: Callable[[], bool]) -> dict:
    torch.cuda.synchronize()
    status, exc_type, message = "rejected", None, None
    try:
        call()
        status = "passed_without_exception"
    except Exception as e:  # noqa: BLE001 - any exception is a rejection
        exc_type = type(e).__name__
        message = str(e).splitlines()[0][:300] if str(e) else ""
    rec = {
        "variant": variant,
        "description": description,
        "expected": expected,
        "status": status,
        "exception_type": exc_type,
        "message": message,
        "expect_msg_contains": expect_msg_contains,
        "msg_match": (expect_msg_contains in message)
        if (expect_msg_contains and message is not None) else None,
        "post_check_ok": None,
    }
    if expected == "skip":
        rec["status"] = "skipped"
        return rec
    rec["post_check_ok"] = bool(control_ok())
    if expected == "reject":
        rec["pass"] = (status == "rejected") and rec["post_check_ok"] and \
            (rec["msg_match"] is not False)
    else:
        rec["pass"] = (status == "passed_without_exception") and rec["post_check_ok"]
    return rec


def summarize_cases(results: list[dict]) -> dict:
    rej = [r for r in results if r["expected"] == "reject"]
    ok = [r for r in results if r["expected"] == "pass"]
    return {
        "n_total": len(results),
        "n_reject_expected": len(rej),
        "n_reject_ok": sum(1 for r in rej if r.get("pass")),
        "n_pass_expected": len(ok),
        "n_pass_ok": sum(1 for r in ok if r.get("pass")),
        "n_skipped": sum(1 for r in results if r["expected"] == "skip"),
        "n_passed": sum(1 for r in results if r.get("pass")),
        "all_pass": all(r.get("pass") for r in results if r["expected"] != "skip"),
    }
