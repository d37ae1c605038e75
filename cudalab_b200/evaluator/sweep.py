"""Shape sweep of the single-GPU GEMV (L2-cold weight pools, CUDA graphs).

The reference times its operators shape by shape with a paired CUDA-event
harness (cudalab/evaluator/bench.py measure_block :259-311) in hot and
streaming modes.  A B200 launch lasts 1-30 us, so here every point is a CUDA
graph of `--launches` GEMVs that cycles through a pool of independently
seeded weight sets larger than three times the L2 cache (or `--pool` sets),
replayed `--reps` times between two events on the launching stream; the
point is the median of `--blocks` such timings.  One JSON line per point:

    python -m cudalab_b200.evaluator.sweep --kinds int4gemv,qgemv \
        --shapes 4096x4096,1024x4096,4096x1024,11008x4096,4096x11008 \
        --batches 1 --flags 3,7

`flags` are the C-ABI launch flags (1 = programmatic dependent launch,
3 = x not produced by the preceding kernel, 7 = neither is y).  GB/s counts
the algorithmic bytes of one GEMV (weights, scales, x, y).  Kinds: int4gemv,
qgemv, gemv (dense fp16) and gemv_f32 (dense fp32; M = 1 only).
"""
from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from cudalab_b200 import _native as nat
from cudalab_b200.build import build
from cudalab_b200.int4gemv_quantize import quantize_w as quantize_int4
from cudalab_b200.operators.gemv import algorithmic_bytes_gemv, make_w
from cudalab_b200.operators.int4gemv import algorithmic_bytes_int4
from cudalab_b200.operators.qgemv import algorithmic_bytes_int8
from cudalab_b200.qgemv_quantize import quantize_w as quantize_int8

ROOT = Path(__file__).resolve().parents[2]
L2_BYTES = 126 * 2**20


def measured_hbm_gbs() -> float | None:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def weight_pool(kind: str, N: int, K: int, pool: int) -> list:
    """(weights, scales) per pool entry; scales are None for the dense GEMV."""
    out = []
    for i in range(pool):
        if kind in ("gemv", "gemv_f32"):
            dt = torch.float16 if kind == "gemv" else torch.float32
            out.append((make_w(N, K, dt, device="cuda", seed=1000 + i, scale=0.02), None))
            continue
        quant = quantize_int4 if kind == "int4gemv" else quantize_int8
        g = torch.Generator().manual_seed(1000 + i)
        W = (torch.randn(N, K, generator=g) * 0.02).half().cuda()
        out.append(quant(W))
        del W
    torch.cuda.synchronize()
    return out


def time_point(ext, variant: str, ws: list, X: torch.Tensor, Y: torch.Tensor, flags: int,
               launches: int, reps: int, blocks: int) -> float:
    """Median over `blocks` of (event time of `reps` graph replays) / GEMVs."""
    M = X.size(0)
    s = torch.cuda.Stream()

    def body():
        for i in range(launches):
            w, sc = ws[i % len(ws)]
            if sc is None:
                ext.forward_into(variant, w, X[0], Y[0], flags=flags)
            elif M == 1:
                ext.forward_into(variant, w, sc, X[0], Y[0], flags=flags)
            else:
                ext.forward_batched_into(variant, w, sc, X, Y, flags=flags)

    with torch.cuda.stream(s):
        body()
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        body()
    times = []
    with torch.cuda.stream(s):
        for _ in range(3):
            g.replay()
        for _ in range(blocks):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(s)
            for _ in range(reps):
                g.replay()
            b.record(s)
            b.synchronize()
            times.append(a.elapsed_time(b) * 1e3 / (reps * launches))
    del g
    return statistics.median(times)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--kinds", default="int4gemv,qgemv")
    ap.add_argument("--shapes", default="4096x4096,1024x4096,4096x1024,11008x4096,4096x11008")
    ap.add_argument("--batches", default="1", help="activation rows M, e.g. 1,4,16")
    ap.add_argument("--flags", default="3,7")
    ap.add_argument("--variant", default="mma", help="variant suffix (int4gemv_<suffix>)")
    ap.add_argument("--pool", type=int, default=0, help="weight sets (0: > 3 x L2)")
    ap.add_argument("--launches", type=int, default=32)
    ap.add_argument("--reps", type=int, default=40)
    ap.add_argument("--blocks", type=int, default=5)
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("sweep needs a CUDA device")
    peak = measured_hbm_gbs()
    exts = {k: build("gemv" if k == "gemv_f32" else k) for k in args.kinds.split(",")}
    for kind, ext in exts.items():
        variant = f"{'gemv' if kind == 'gemv_f32' else kind}_{args.variant}"
        es = 4 if kind == "gemv_f32" else 2
        bytes_fn = {"int4gemv": algorithmic_bytes_int4, "qgemv": algorithmic_bytes_int8,
                    "gemv": lambda N, K, M: algorithmic_bytes_gemv(N, K, es) if M else N * K * es,
                    "gemv_f32": lambda N, K, M: algorithmic_bytes_gemv(N, K, es) if M
                    else N * K * es}[kind]
        for shape in args.shapes.split(","):
            N, K = (int(v) for v in shape.lower().split("x"))
            wbytes = bytes_fn(N, K, 0)
            pool = args.pool or max(2, -(-3 * L2_BYTES // wbytes))
            ws = weight_pool(kind, N, K, pool)
            xdt = torch.float32 if kind == "gemv_f32" else torch.float16
            for M in (int(m) for m in args.batches.split(",")):
                if kind.startswith("gemv") and M != 1:
                    continue
                X = torch.randn(M, K, generator=torch.Generator().manual_seed(7)).to(xdt).cuda()
                Y = torch.empty(M, N, device="cuda", dtype=xdt)
                torch.cuda.synchronize()
                for flags in (int(f) for f in args.flags.split(",")):
                    us = time_point(ext, variant, ws, X, Y, flags, args.launches, args.reps,
                                    args.blocks)
                    gbs = bytes_fn(N, K, M) / (us * 1e-6) / 1e9
                    print(json.dumps({
                        "kind": kind, "variant": variant, "N": N, "K": K, "M": M,
                        "flags": flags, "pool": pool, "us_per_gemv": round(us, 3),
                        "gbs": round(gbs, 1),
                        "frac_of_measured_hbm": round(gbs / peak, 4) if peak else None,
                        "device_status": nat.device_status(clear=True),
                    }), flush=True)
            del ws
            torch.cuda.empty_cache()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
