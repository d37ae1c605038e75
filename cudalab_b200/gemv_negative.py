"""Dense GEMV negative suite: 24 per-variant cases (the case table of
cudalab/gemv_negative.py:80-300 of the reference).

Illegal inputs must be rejected before any launch with a message whose first
line carries the pinned substring; legal-but-unaligned inputs (a W view 4
bytes past a 16-byte boundary, x 2 bytes past) must run, and a vectorised
variant given them, or K = 13, must return exactly what `gemv_baseline`
returns (its fallback).  The quarantined `gemv_splitk4` has no alignment
contract (scalar loads): its two misaligned cases only require a finite,
unrejected result, and only K = 13 (its contract K % 4 == 0 unmet) must
match the baseline.  After every case a control forward checks the context.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

from .evaluator.negative import run_case as _run_case, summarize_cases
from .operators.gemv import make_w, make_x

SUITE_VERSION = "negative-gemv-b200"
V = "gemv_baseline"


def _post_check_ok(ext, variant: str = V) -> bool:
    try:
        torch.cuda.synchronize()
        W = torch.randn(2, 16, dtype=torch.float16, device="cuda")
        x = torch.randn(16, dtype=torch.float16, device="cuda")
        y = ext.forward(variant, W, x)
        torch.cuda.synchronize()
        return bool(torch.isfinite(y.float()).all())
    except Exception:  # noqa: BLE001
        return False


def build_cases(ext, variant: str = V) -> list[dict]:
    dev = "cuda"
    cases: list[dict] = []

    def add(cid, desc, call, expected="reject", msg=None):
        cases.append(dict(id=cid, variant=variant, description=desc, call=call,
                          expected=expected, expect_msg_contains=msg))

    N, K = 8, 64
    W = make_w(N, K, torch.float16, device=dev, seed=0)
    x = make_x(K, torch.float16, device=dev, seed=0)

    def fwd(a, b):
        return ext.forward(variant, a, b)

    # ---- W ----
    w1d = torch.randn(N * K, dtype=torch.float16, device=dev)
    add("W_1d", "W is 1-D (N*K,)", lambda: fwd(w1d, x), msg="必须是 2 维")
    w3d = torch.randn(2, 4, 8, dtype=torch.float16, device=dev)
    add("W_3d", "W is 3-D (2, 4, 8)", lambda: fwd(w3d, x), msg="必须是 2 维")
    wn0 = torch.empty(0, K, dtype=torch.float16, device=dev)
    add("W_N_zero", "N == 0", lambda: fwd(wn0, x), msg="N 必须 > 0")
    wk0 = torch.empty(N, 0, dtype=torch.float16, device=dev)
    add("W_K_zero", "K == 0", lambda: fwd(wk0, x), msg="K 必须 > 0")
    wbf = make_w(N, K, torch.bfloat16, device=dev, seed=0)
    add("W_bfloat16", "W bfloat16 (fp16 / fp32 only)", lambda: fwd(wbf, x),
        msg="float16 / float32")
    wi = torch.randint(-3, 3, (N, K), dtype=torch.int32, device=dev)
    add("W_int32", "W int32", lambda: fwd(wi, x), msg="float16 / float32")
    wcpu = make_w(N, K, torch.float16, device="cpu", seed=0)
    add("W_cpu", "W on the CPU", lambda: fwd(wcpu, x), msg="CUDA 张量")
    wt = make_w(K, N, torch.float16, device=dev, seed=1).t()
    add("W_transpose_view", "W a transposed (K, N) view", lambda: fwd(wt, x), msg="连续内存")
    add("unknown_variant", "unknown variant name",
        lambda: ext.forward("no_such_gemv_variant", W, x), msg="未知 gemv 变体")

    # ---- x ----
    x_short = make_x(K - 1, torch.float16, device=dev, seed=2)
    add("x_len_mismatch", "len(x) = 63 != K = 64", lambda: fwd(W, x_short), msg="长度必须等于 K")
    add("x_2d", "x is 2-D (1, 64)", lambda: fwd(W, x.view(1, K)), msg="必须是 1 维")
    x32 = make_x(K, torch.float32, device=dev, seed=3)
    add("x_dtype_mismatch", "x float32, W float16", lambda: fwd(W, x32), msg="dtype 必须与 W 一致")
    xcpu = make_x(K, torch.float16, device="cpu", seed=4)
    add("x_cpu", "x on the CPU", lambda: fwd(W, xcpu), msg="CUDA 张量")
    x_nc = torch.randn(2 * K, dtype=torch.float16, device=dev)[::2]
    add("x_noncontiguous", "x a stride-2 slice", lambda: fwd(W, x_nc), msg="连续内存")

    # ---- out of forward_into ----
    add("out_wrong_shape", "len(out) = 7 != N = 8",
        lambda: ext.forward_into(variant, W, x, torch.empty(N - 1, dtype=torch.float16,
                                                            device=dev)),
        msg="长度必须等于 N")
    add("out_wrong_dtype", "out float32, W float16",
        lambda: ext.forward_into(variant, W, x, torch.empty(N, dtype=torch.float32, device=dev)),
        msg="dtype 必须与 W 一致")
    o_nc = torch.randn(2 * N, dtype=torch.float16, device=dev)[::2]
    add("out_noncontiguous", "out a stride-2 slice",
        lambda: ext.forward_into(variant, W, x, o_nc), msg="连续内存")
    add("out_cpu", "out on the CPU",
        lambda: ext.forward_into(variant, W, x, torch.empty(N, dtype=torch.float16)),
        msg="CUDA 张量")

    # ---- controls: legal inputs must not be rejected ----
    out_ok = torch.empty(N, dtype=torch.float16, device=dev)
    add("valid_forward_into_control", "legal forward_into",
        lambda: ext.forward_into(variant, W, x, out_ok), expected="pass")
    big_w = torch.randn(N * K + 2, dtype=torch.float16, device=dev)
    w_off = big_w[2:2 + N * K].view(N, K)          # base 4 bytes past 16-byte alignment
    x_ok = make_x(K, torch.float16, device=dev, seed=5)

    def _offset_control():
        ext.forward_into(variant, w_off, x_ok, out_ok)
        y = ext.forward(variant, W, x)
        assert bool(torch.isfinite(out_ok.float()).all()), "offset-view output not finite"
        assert bool(torch.isfinite(y.float()).all()), "control output not finite"

    add("valid_offset_view_control", "W contiguous view 4 bytes off a 16-byte boundary must run",
        _offset_control, expected="pass")
    x_off = torch.randn(K + 1, dtype=torch.float16, device=dev)[1:1 + K]
    add("valid_offset_view_x", "x 2 bytes off a 16-byte boundary must run",
        lambda: fwd(W, x_off), expected="pass")

    # ---- fallback bit-identity against the baseline ----
    def _fallback_check(tag, Wm, xm, n_rows):
        out_f = torch.empty(n_rows, dtype=torch.float16, device=dev)
        ext.forward_into(variant, Wm, xm, out_f)
        torch.cuda.synchronize()
        y_base = ext.forward("gemv_baseline", Wm, xm)
        torch.cuda.synchronize()
        assert torch.equal(out_f, y_base), f"{tag}: fallback output differs from gemv_baseline"

    def _finite_control(Wm, xm, tag):
        out_f = torch.empty(N, dtype=torch.float16, device=dev)
        ext.forward_into(variant, Wm, xm, out_f)
        torch.cuda.synchronize()
        assert bool(torch.isfinite(out_f.float()).all()), f"{tag}: output not finite"

    wm = torch.randn(N * K + 2, dtype=torch.float16, device=dev)[2:2 + N * K].view(N, K)
    xa = make_x(K, torch.float16, device=dev, seed=6)
    wa = make_w(N, K, torch.float16, device=dev, seed=7)
    xm = torch.randn(K + 1, dtype=torch.float16, device=dev)[1:1 + K]
    if variant == "gemv_splitk4":
        add("fallback_W_misaligned", "splitk4 (no alignment contract): misaligned W runs, finite",
            lambda: _finite_control(wm, xa, "W misaligned"), expected="pass")
        add("fallback_x_misaligned", "splitk4 (no alignment contract): misaligned x runs, finite",
            lambda: _finite_control(wa, xm, "x misaligned"), expected="pass")
    else:
        add("fallback_W_misaligned", "W not 16-byte aligned: baseline fallback, bit-identical",
            lambda: _fallback_check("fallback_W_misaligned", wm, xa, N), expected="pass")
        add("fallback_x_misaligned", "x not 16-byte aligned: baseline fallback, bit-identical",
            lambda: _fallback_check("fallback_x_misaligned", wa, xm, N), expected="pass")
    wk = make_w(16, 13, torch.float16, device=dev, seed=8)
    xk = make_x(13, torch.float16, device=dev, seed=9)
    add("fallback_K_not_mult8", "K = 13: baseline fallback, bit-identical",
        lambda: _fallback_check("fallback_K_not_mult8", wk, xk, 16), expected="pass")
    return cases


def run_negative_suite(ext, out_path: Path | None = None, variant: str = V) -> dict:
    results = []
    for c in build_cases(ext, variant):
        r = _run_case(c["variant"], c["description"], c["call"], c["expected"],
                      c["expect_msg_contains"], lambda v=c["variant"]: _post_check_ok(ext, v))
        r["id"] = c["id"]
        results.append(r)
    doc = {"suite": SUITE_VERSION, "negative_suite_scope": "per-variant",
           "summary": summarize_cases(results), "cases": results}
    if out_path is not None:
        Path(out_path).parent.mkdir(parents=True, exist_ok=True)
        Path(out_path).write_text(json.dumps(doc, indent=2, ensure_ascii=False))
    return doc
