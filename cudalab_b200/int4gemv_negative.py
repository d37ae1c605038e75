"""INT4 GEMV negative suite: 30 per-variant cases
(the case table of cudalab/int4gemv_negative.py:92-319).

Illegal inputs must be rejected before any launch with a message whose first
line carries the pinned substring; legal-but-unaligned inputs (1-byte offset
W_packed view, 2-byte offset x) must run, and a vectorised variant given them
must produce output bit-identical to `int4gemv_baseline` (its scalar
fallback).  After every case a control forward checks the context is healthy.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

from .evaluator.negative import run_case as _run_case, summarize_cases
from .operators.int4gemv import make_w4, make_x4

SUITE_VERSION = "negative-int4gemv-b200"
V = "int4gemv_baseline"


def _post_check_ok(ext, variant: str = V) -> bool:
    try:
        torch.cuda.synchronize()
        Wp, s, _ = make_w4(2, 128, seed=0)
        x = make_x4(128, seed=1)
        y = ext.forward(variant, Wp, s, x)
        torch.cuda.synchronize()
        return bool(torch.isfinite(y.float()).all())
    except Exception:  # noqa: BLE001
        return False


def _rand_bytes(shape, seed: int, device: str = "cuda") -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(0, 256, shape, generator=g, dtype=torch.uint8).to(device)


def build_cases(ext, variant: str = V) -> list[dict]:
    dev = "cuda"
    cases: list[dict] = []

    def add(cid, desc, call, expected="reject", msg=None):
        cases.append(dict(id=cid, variant=variant, description=desc, call=call,
                          expected=expected, expect_msg_contains=msg))

    N, K = 8, 256
    Wp, s, _ = make_w4(N, K, seed=0)
    x = make_x4(K, seed=1)

    def fwd(a, b, c):
        return ext.forward(variant, a, b, c)

    # ---- W_packed ----
    w1d = _rand_bytes((N * K // 2,), 2)
    add("W_packed_1d", "W_packed is 1-D", lambda: fwd(w1d, s, x), msg="必须是 2 维")
    w3d = _rand_bytes((N, K // 2), 3).view(2, N // 2, K // 2)
    add("W_packed_3d", "W_packed is 3-D", lambda: fwd(w3d, s, x), msg="必须是 2 维")
    wn0 = torch.empty(0, K // 2, dtype=torch.uint8, device=dev)
    add("W_packed_N_zero", "N == 0", lambda: fwd(wn0, s[:0].contiguous(), x), msg="N 必须 > 0")
    wk0 = torch.empty(N, 0, dtype=torch.uint8, device=dev)
    add("W_packed_K2_zero", "K/2 == 0", lambda: fwd(wk0, s, x), msg="K/2 必须 > 0")
    wf16 = torch.randn(N, K // 2, dtype=torch.float16, device=dev)
    add("W_packed_dtype_fp16", "W_packed fp16", lambda: fwd(wf16, s, x), msg="必须是 uint8")
    wi8 = _rand_bytes((N, K // 2), 12).to(torch.int8)
    add("W_packed_dtype_int8", "W_packed int8", lambda: fwd(wi8, s, x), msg="必须是 uint8")
    wcpu = _rand_bytes((N, K // 2), 4, device="cpu")
    add("W_packed_cpu", "W_packed on the CPU", lambda: fwd(wcpu, s.cpu(), x.cpu()),
        msg="CUDA 张量")
    wt = _rand_bytes((K, N // 2), 5).t()
    add("W_packed_noncontig", "W_packed transposed view", lambda: fwd(wt, s, x), msg="连续内存")

    # ---- K % 128 contract (hard rejection, before any scale check) ----
    wk64 = _rand_bytes((N, 32), 6)
    add("K_not_mult128", "K = 64",
        lambda: fwd(wk64, torch.zeros(N, 1, dtype=torch.float16, device=dev),
                    make_x4(64, seed=6)),
        msg="必须可被 128 整除")

    # ---- scale ----
    s_short = s[:, :s.size(1) - 1].contiguous()
    add("scale_group_count", "scale has K/128 - 1 groups", lambda: fwd(Wp, s_short, x),
        msg="scale 组数必须等于 K/128")
    s_nshort = s[:N - 1].contiguous()
    add("scale_N_mismatch", "scale has N - 1 rows", lambda: fwd(Wp, s_nshort, x),
        msg="scale 行数必须等于 N")
    add("scale_1d", "scale is 1-D", lambda: fwd(Wp, s.view(-1), x), msg="必须是 2 维")
    add("scale_dtype_fp32", "scale fp32", lambda: fwd(Wp, s.float(), x), msg="必须是 float16")
    add("scale_cpu", "scale on the CPU", lambda: fwd(Wp, s.cpu(), x), msg="CUDA 张量")
    s_nc = torch.randn(2 * N, s.size(1), dtype=torch.float16, device=dev)[::2]
    add("scale_noncontig", "scale row-strided view", lambda: fwd(Wp, s_nc, x), msg="连续内存")

    # ---- x ----
    x_short = make_x4(K - 128, seed=7)
    add("x_len_mismatch", "len(x) = K - 128", lambda: fwd(Wp, s, x_short),
        msg="x 长度必须等于 K")
    add("x_2d", "x is (1, K)", lambda: fwd(Wp, s, x.view(1, K)), msg="必须是 1 维")
    x32 = make_x4(K, seed=8).float()
    add("x_dtype_fp32", "x fp32", lambda: fwd(Wp, s, x32), msg="必须是 float16")
    add("x_cpu", "x on the CPU", lambda: fwd(Wp, s, x.cpu()), msg="CUDA 张量")
    x_nc = torch.randn(2 * K, dtype=torch.float16, device=dev)[::2]
    add("x_noncontig", "x strided view", lambda: fwd(Wp, s, x_nc), msg="连续内存")

    # ---- out (forward_into) ----
    add("out_wrong_shape", "len(out) = N - 1",
        lambda: ext.forward_into(variant, Wp, s, x,
                                 torch.empty(N - 1, dtype=torch.float16, device=dev)),
        msg="out 长度必须等于 N")
    add("out_wrong_dtype", "out fp32",
        lambda: ext.forward_into(variant, Wp, s, x,
                                 torch.empty(N, dtype=torch.float32, device=dev)),
        msg="必须是 float16")
    o_nc = torch.randn(2 * N, dtype=torch.float16, device=dev)[::2]
    add("out_noncontig", "out strided view",
        lambda: ext.forward_into(variant, Wp, s, x, o_nc), msg="连续内存")
    add("out_cpu", "out on the CPU",
        lambda: ext.forward_into(variant, Wp, s, x, torch.empty(N, dtype=torch.float16)),
        msg="CUDA 张量")

    # ---- variant name ----
    add("unknown_variant", "unknown variant name",
        lambda: ext.forward("no_such_int4gemv_variant", Wp, s, x), msg="未知 int4gemv 变体")

    # ---- controls: legal inputs must not be rejected ----
    out_ok = torch.empty(N, dtype=torch.float16, device=dev)
    add("valid_forward_into_control", "legal forward_into",
        lambda: ext.forward_into(variant, Wp, s, x, out_ok), expected="pass")
    big_wp = _rand_bytes((N * K // 2 + 1,), 9)
    wp_mis = big_wp[1:1 + N * K // 2].view(N, K // 2)   # base offset 1 byte

    def _wp_offset_control():
        ext.forward_into(variant, wp_mis, s, x, out_ok)
        y = ext.forward(variant, Wp, s, x)
        assert bool(torch.isfinite(out_ok.float()).all()), "offset-view output not finite"
        assert bool(torch.isfinite(y.float()).all()), "control output not finite"

    add("valid_offset_view_Wp_control", "W_packed 1-byte offset contiguous view must run",
        _wp_offset_control, expected="pass")
    x_mis = torch.randn(K + 1, dtype=torch.float16, device=dev)[1:1 + K]  # 2-byte offset
    add("valid_offset_view_x_control", "x 2-byte offset view must run",
        lambda: fwd(Wp, s, x_mis), expected="pass")

    # ---- fallback bit-identity against the baseline ----
    def _fallback_check(tag, Wm, xm):
        out_f = torch.empty(N, dtype=torch.float16, device=dev)
        ext.forward_into(variant, Wm, s, xm, out_f)
        torch.cuda.synchronize()
        y_base = ext.forward("int4gemv_baseline", Wm, s, xm)
        torch.cuda.synchronize()
        assert torch.equal(out_f, y_base), f"{tag}: fallback output differs from int4gemv_baseline"

    xa = make_x4(K, seed=10)
    Wa, _, _ = make_w4(N, K, seed=11)
    xm = torch.randn(K + 1, dtype=torch.float16, device=dev)[1:1 + K]
    add("fallback_Wp_misaligned", "W_packed not 16-byte aligned: scalar fallback, bit-identical",
        lambda: _fallback_check("fallback_Wp_misaligned", wp_mis, xa), expected="pass")
    add("fallback_x_misaligned", "x not 16-byte aligned: scalar fallback, bit-identical",
        lambda: _fallback_check("fallback_x_misaligned", Wa, xm), expected="pass")
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
