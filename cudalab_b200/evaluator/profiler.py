"""ncu wrapper (role of cudalab/evaluator/profiler.py:145-336) for B200.

Runs `ncu --csv` on a small, self-terminating driver in a subprocess and
parses the per-launch metrics into a summary.  Always passes
`--clock-control none` (the GPU's clocks are never locked) and profiles one
kernel (`-k`), a handful of launches (`-c`).  Adds the metrics the reference's
list lacked: dram__bytes_read.sum / dram__bytes_write.sum (physical DRAM
traffic per launch, compared against the algorithmic bytes) and the tensor /
issue counters that tell whether a kernel is bound by instruction issue.

    python -m cudalab_b200.evaluator.profiler --op int4gemv --variant int4gemv_bulk \
        --N 4096 --K 4096 --out prof_int4_bulk.json
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import shutil
import subprocess
import sys
from pathlib import Path

METRICS = [
    "gpu__time_duration.sum",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "dram__throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__cycles_elapsed.avg",
    "smsp__cycles_active.avg",
    "smsp__inst_executed.sum",
    "smsp__issue_active.avg.pct_of_peak_sustained_active",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "sm__inst_executed_pipe_alu.sum",
    "sm__inst_executed_pipe_fma.sum",
    "sm__inst_executed_pipe_fmaheavy.sum",
    "sm__inst_executed_pipe_fmalite.sum",
    "sm__inst_executed_pipe_fma_type_fp16.sum",
    "sm__inst_executed_pipe_lsu.sum",
    "sm__inst_executed_pipe_uniform.sum",
    "sm__inst_executed_pipe_xu.sum",
    "sm__inst_executed_pipe_tensor.sum",
    "sm__pipe_alu_cycles_active.avg.pct_of_peak_sustained_active",
    "sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_active",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "l1tex__data_pipe_lsu_wavefronts_mem_shared.sum",
    "launch__registers_per_thread",
    "launch__grid_size",
    "launch__block_size",
    "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_short_scoreboard_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_barrier_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_wait_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_math_pipe_throttle_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_not_selected_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_selected_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_dispatch_stall_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_mio_throttle_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_lg_throttle_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_no_instruction_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_sleeping_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_membar_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_drain_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_branch_resolving_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_misc_per_issue_active.ratio",
]

ROOT = Path(__file__).resolve().parents[2]


def driver_main(argv=None) -> int:
    """The profiled program: builds a small L2-cold pool and launches each
    weight set once (ncu flushes caches before every replay pass anyway).
    --M > 1 launches the batched entry point with M activation rows."""
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="int4gemv")
    ap.add_argument("--variant", default="int4gemv_bulk")
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--pool", type=int, default=4)
    ap.add_argument("--launches", type=int, default=6)
    ap.add_argument("--pdl", type=int, default=0)
    ap.add_argument("--rmsnorm", action="store_true",
                    help="fused RMSNorm -> INT4 GEMV (variant int4gemv_rmsnorm*), M rows")
    a = ap.parse_args(argv)
    sys.path.insert(0, str(ROOT))
    import torch
    from cudalab_b200.build import build
    from cudalab_b200.operators import get
    op = get(a.op)
    ext = build(a.op)
    pool = op.make_bench_pool(a.N, a.K, mode="l2cold", pool_size=a.pool, weight_dist=0.02)
    if a.rmsnorm:
        X = torch.randn(a.M, a.K, device="cuda").half()
        gw = (torch.randn(a.K, device="cuda") * 0.5 + 1.0).half()
        Y = torch.empty(a.M, a.N, device="cuda", dtype=torch.float16)
        weights = pool.shared["weights"]
        for i in range(a.launches):
            W, s = weights[i % len(weights)]
            ext.forward_rmsnorm(a.variant, W, s, X, gw, out=Y, flags=a.pdl)
    elif a.M == 1:
        for i in range(a.launches):
            pool.launch(ext, a.variant, i, flags=a.pdl)
    else:
        X = torch.randn(a.M, a.K, device="cuda").half()
        Y = torch.empty(a.M, a.N, device="cuda", dtype=torch.float16)
        weights = pool.shared["weights"]
        for i in range(a.launches):
            W, s = weights[i % len(weights)]
            ext.forward_batched_into(a.variant, W, s, X, Y, flags=a.pdl)
    torch.cuda.synchronize()
    print("profile driver done", a.variant, a.N, a.K, a.M)
    return 0


def parse_csv(text: str) -> list[dict]:
    """ncu --csv (long format, one row per metric) -> one dict per launch."""
    lines = [ln for ln in text.splitlines() if ln.startswith('"')]
    if not lines:
        return []
    rows = list(csv.DictReader(io.StringIO("\n".join(lines))))
    launches: dict = {}
    for r in rows:
        key = r.get("ID")
        d = launches.setdefault(key, {"id": key, "kernel": r.get("Kernel Name"), "metrics": {}})
        name, val, unit = r.get("Metric Name"), r.get("Metric Value"), r.get("Metric Unit")
        try:
            v = float(str(val).replace(",", ""))
        except (TypeError, ValueError):
            v = val
        d["metrics"][name] = {"value": v, "unit": unit}
    return list(launches.values())


def profile(op: str, variant: str, N: int, K: int, out: Path, kernel_regex: str,
            launch_skip: int = 2, launch_count: int = 3, ncu: str | None = None) -> dict:
    ncu = ncu or shutil.which("ncu") or "/usr/local/cuda/bin/ncu"
    cmd = [ncu, "--csv", "--clock-control", "none", "-k", f"regex:{kernel_regex}",
           "-s", str(launch_skip), "-c", str(launch_count), "--metrics", ",".join(METRICS),
           sys.executable, "-m", "cudalab_b200.evaluator.profiler", "--driver",
           "--op", op, "--variant", variant, "--N", str(N), "--K", str(K)]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=str(ROOT))
    launches = parse_csv(proc.stdout)
    summary = {"variant": variant, "op": op, "shape": [N, K], "cmd": " ".join(cmd),
               "returncode": proc.returncode, "launches": launches}
    if launches:
        m = launches[-1]["metrics"]
        rd = m.get("dram__bytes_read.sum", {}).get("value")
        wr = m.get("dram__bytes_write.sum", {}).get("value")
        if isinstance(rd, float) and isinstance(wr, float):
            summary["traffic_bytes_per_launch"] = int(rd + wr)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(summary, indent=2))
    if proc.returncode != 0:
        (out.with_suffix(".stderr.txt")).write_text(proc.stdout[-4000:] + proc.stderr[-4000:])
    return summary


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if "--driver" in argv:
        argv.remove("--driver")
        return driver_main(argv)
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="int4gemv")
    ap.add_argument("--variant", default="int4gemv_bulk")
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--kernel-regex", default="gemv")
    ap.add_argument("--out", type=Path, required=True)
    a = ap.parse_args(argv)
    s = profile(a.op, a.variant, a.N, a.K, a.out, a.kernel_regex)
    print(json.dumps({k: v for k, v in s.items() if k != "launches"}, indent=2))
    return 0 if s["returncode"] == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
