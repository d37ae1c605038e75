"""INT8 GEMV negative suite: 29 per-variant cases
(the case table of cudalab/qgemv_negative.py:104-296), including the INT8-only
`fallback_K_not_mult16` (K = 13 must run the scalar fallback bit-identically).
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

from .evaluator.negative import run_case as _run_case, summarize_cases
from .operators.qgemv import make_w_q, make_x_q

SUITE_VERSION = "negative-qgemv-b200"
V = "qgemv_baseline"


def _post_check_ok(ext, variant: str = V) -> bool:
    try:
        torch.cuda.synchronize()
        Wq, s, _ = make_w_q(2, 16, seed=0)
        x = make_x_q(16, seed=1)
        y = ext.forward(variant, Wq, s, x)
        torch.cuda.synchronize()
        return bool(torch.isfinite(y.float()).all())
    except Exception:  # noqa: BLE001
        return False


def _rand_q(shape, seed: int, device: str = "cuda") -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(-127, 128, shape, generator=g, dtype=torch.int8).to(device)


def build_cases(ext, variant: str = V) -> list[dict]:
    dev = "cuda"
    cases: list[dict] = []

    def add(cid, desc, call, expected="reject", msg=None):
        cases.append(dict(id=cid, variant=variant, description=desc, call=call,
                          expected=expected, expect_msg_contains=msg))

    N, K = 8, 64
    Wq, s, _ = make_w_q(N, K, seed=0)
    x = make_x_q(K, seed=1)

    def fwd(a, b, c):
        return ext.forward(variant, a, b, c)

    # ---- W_q ----
    w1d = _rand_q((N * K,), 2)
    add("W_q_1d", "W_q is 1-D", lambda: fwd(w1d, s, x), msg="必须是 2 维")
    w3d = _rand_q((N, K), 3).view(2, N // 2, K)
    add("W_q_3d", "W_q is 3-D", lambda: fwd(w3d, s, x), msg="必须是 2 维")
    wn0 = torch.empty(0, K, dtype=torch.int8, device=dev)
    add("W_q_N_zero", "N == 0", lambda: fwd(wn0, s[:0].contiguous(), x), msg="N 必须 > 0")
    wk0 = torch.empty(N, 0, dtype=torch.int8, device=dev)
    add("W_q_K_zero", "K == 0", lambda: fwd(wk0, s, x), msg="K 必须 > 0")
    wf = torch.randn(N, K, dtype=torch.float16, device=dev)
    add("W_q_dtype_fp16", "W_q fp16", lambda: fwd(wf, s, x), msg="必须是 int8")
    wi = torch.randint(-3, 3, (N, K), dtype=torch.int32, device=dev)
    add("W_q_dtype_int32", "W_q int32", lambda: fwd(wi, s, x), msg="必须是 int8")
    wcpu = _rand_q((N, K), 4, device="cpu")
    add("W_q_cpu", "W_q on the CPU", lambda: fwd(wcpu, s.cpu(), x.cpu()), msg="CUDA 张量")
    wt = _rand_q((K, N), 5).t()
    add("W_q_noncontig", "W_q transposed view", lambda: fwd(wt, s, x), msg="连续内存")

    # ---- scale ----
    add("scale_len_mismatch", "len(scale) = N - 1", lambda: fwd(Wq, s[:N - 1].contiguous(), x),
        msg="scale 长度必须等于 N")
    add("scale_2d", "scale is (N, 1)", lambda: fwd(Wq, s.view(N, 1), x), msg="必须是 1 维")
    add("scale_dtype_fp16", "scale fp16", lambda: fwd(Wq, s.half(), x), msg="必须是 float32")
    add("scale_cpu", "scale on the CPU", lambda: fwd(Wq, s.cpu(), x), msg="CUDA 张量")
    s_nc = torch.rand(2 * N, dtype=torch.float32, device=dev)[::2]
    add("scale_noncontig", "scale strided view", lambda: fwd(Wq, s_nc, x), msg="连续内存")

    # ---- x ----
    add("x_len_mismatch", "len(x) = K - 1", lambda: fwd(Wq, s, make_x_q(K - 1, seed=6)),
        msg="x 长度必须等于 K")
    add("x_2d", "x is (1, K)", lambda: fwd(Wq, s, x.view(1, K)), msg="必须是 1 维")
    add("x_dtype_fp32", "x fp32", lambda: fwd(Wq, s, make_x_q(K, seed=7).float()),
        msg="必须是 float16")
    add("x_cpu", "x on the CPU", lambda: fwd(Wq, s, x.cpu()), msg="CUDA 张量")
    x_nc = torch.randn(2 * K, dtype=torch.float16, device=dev)[::2]
    add("x_noncontig", "x strided view", lambda: fwd(Wq, s, x_nc), msg="连续内存")

    # ---- out ----
    add("out_wrong_shape", "len(out) = N - 1",
        lambda: ext.forward_into(variant, Wq, s, x,
                                 torch.empty(N - 1, dtype=torch.float16, device=dev)),
        msg="out 长度必须等于 N")
    add("out_wrong_dtype", "out fp32",
        lambda: ext.forward_into(variant, Wq, s, x,
                                 torch.empty(N, dtype=torch.float32, device=dev)),
        msg="必须是 float16")
    o_nc = torch.randn(2 * N, dtype=torch.float16, device=dev)[::2]
    add("out_noncontig", "out strided view", lambda: ext.forward_into(variant, Wq, s, x, o_nc),
        msg="连续内存")
    add("out_cpu", "out on the CPU",
        lambda: ext.forward_into(variant, Wq, s, x, torch.empty(N, dtype=torch.float16)),
        msg="CUDA 张量")

    add("unknown_variant", "unknown variant name",
        lambda: ext.forward("no_such_qgemv_variant", Wq, s, x), msg="未知 qgemv 变体")

    # ---- controls ----
    out_ok = torch.empty(N, dtype=torch.float16, device=dev)
    add("valid_forward_into_control", "legal forward_into",
        lambda: ext.forward_into(variant, Wq, s, x, out_ok), expected="pass")
    big = _rand_q((N * K + 1,), 8)
    wq_mis = big[1:1 + N * K].view(N, K)

    def _wq_offset_control():
        ext.forward_into(variant, wq_mis, s, x, out_ok)
        y = ext.forward(variant, Wq, s, x)
        assert bool(torch.isfinite(out_ok.float()).all()), "offset-view output not finite"
        assert bool(torch.isfinite(y.float()).all()), "control output not finite"

    add("valid_offset_view_Wq_control", "W_q 1-byte offset view must run", _wq_offset_control,
        expected="pass")
    x_mis = torch.randn(K + 1, dtype=torch.float16, device=dev)[1:1 + K]
    add("valid_offset_view_x_control", "x 2-byte offset view must run",
        lambda: fwd(Wq, s, x_mis), expected="pass")

    # ---- fallback bit-identity ----
    def _fallback_check(tag, Wm, sm, xm, n):
        out_f = torch.empty(n, dtype=torch.float16, device=dev)
        ext.forward_into(variant, Wm, sm, xm, out_f)
        torch.cuda.synchronize()
        y_base = ext.forward("qgemv_baseline", Wm, sm, xm)
        torch.cuda.synchronize()
        assert torch.equal(out_f, y_base), f"{tag}: fallback output differs from qgemv_baseline"

    xa = make_x_q(K, seed=9)
    Wa, sa, _ = make_w_q(N, K, seed=10)
    xm = torch.randn(K + 1, dtype=torch.float16, device=dev)[1:1 + K]
    add("fallback_Wq_misaligned", "W_q not 16-byte aligned: fallback, bit-identical",
        lambda: _fallback_check("fallback_Wq_misaligned", wq_mis, s, xa, N), expected="pass")
    add("fallback_x_misaligned", "x not 16-byte aligned: fallback, bit-identical",
        lambda: _fallback_check("fallback_x_misaligned", Wa, sa, xm, N), expected="pass")
    Wk, sk, _ = make_w_q(16, 13, seed=11)
    xk = make_x_q(13, seed=12)
    add("fallback_K_not_mult16", "K = 13: fallback, bit-identical",
        lambda: _fallback_check("fallback_K_not_mult16", Wk, sk, xk, 16), expected="pass")
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
