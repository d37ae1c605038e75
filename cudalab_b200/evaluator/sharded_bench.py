"""Row-sharded GEMV benchmark (70B-class MLP shapes) over 1/2/4/8 GPUs.

Run one process per GPU:
    python -m torch.distributed.run --nnodes=1 --nproc-per-node G \\
        --master-addr 127.0.0.1 --master-port 29541 \\
        -m cudalab_b200.evaluator.sharded_bench [--kinds int4gemv,qgemv]

Per case (N, K), mode ("fused": peer-store all-gather inside the GEMV;
"nccl": GEMV + NCCL all_gather_into_tensor) and launch flags, every rank holds
a pool of independently seeded weight shards whose total exceeds the L2 cache
(so every step streams its shard from HBM), a graph of L steps cycling through
the pool is captured once and replayed; the step time is the max over ranks of
CUDA-event time / steps.  Reported: us per step, aggregate algorithmic GB/s
(bytes of the full matrix + x + y per step / step time) and its fraction of
world x the measured per-GPU HBM copy bandwidth.  Rank 0 prints one JSON line
per measurement.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from cudalab_b200 import _native as nat  # noqa: E402
from cudalab_b200.operators.int4gemv import algorithmic_bytes_int4  # noqa: E402
from cudalab_b200.operators.qgemv import algorithmic_bytes_int8  # noqa: E402
from cudalab_b200.sharded import PeerBuffers, ShardedGemv, shard_rows  # noqa: E402

L2_BYTES = 126 * 2**20


def hbm_peak() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"])
    return 6650.0


def make_shard(kind, N, K, row0, n, seed, dev):
    """Rows [row0, row0+n) of a seeded full matrix, quantised on the device
    (quantisation is per row / per row group, so it commutes with slicing)."""
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(n, K, generator=g) * 0.02).half().to(dev)
    if kind == "int4gemv":
        from cudalab_b200.int4gemv_quantize import quantize_w
    else:
        from cudalab_b200.qgemv_quantize import quantize_w
    return quantize_w(W)


def time_steps(ops, x, flags, steps, reps, dev):
    """Capture `steps` steps cycling through `ops` into a graph, replay it
    `reps` times; returns (max-over-ranks us per step, max device status)."""
    pool = len(ops)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for i in range(steps):
            ops[i % pool].forward(x, flags=flags)
    st.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(steps):
            ops[i % pool].forward(x, flags=flags)
    with torch.cuda.stream(st):
        for _ in range(2):
            g.replay()
    st.synchronize()
    dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        e0.record(st)
        for _ in range(reps):
            g.replay()
        e1.record(st)
    e1.synchronize()
    us = torch.tensor([e0.elapsed_time(e1) * 1e3 / (reps * steps)], dtype=torch.float64,
                      device=dev)
    dist.all_reduce(us, op=dist.ReduceOp.MAX)
    stat = torch.tensor([nat.device_status(clear=True)], dtype=torch.int32, device=dev)
    dist.all_reduce(stat, op=dist.ReduceOp.MAX)
    del g
    return float(us.item()), int(stat.item())


# ---------------------------------------------------------------------------
# Config 4 of the north-star workload at the run's world size: the 70B-class
# MLP shapes, INT4 G=128, M in {1, 4, 16}, fused and NCCL completion, with
# an in-run parity check.  bench.py calls config4_block on every rank.
# ---------------------------------------------------------------------------
CONFIG4_SHAPES = ((28672, 8192), (8192, 28672))
CONFIG4_BATCHES = (1, 4, 16)
CONFIG4_FLAGS = 3  # PDL | inputs ready: x is replicated and not produced by the step before


def _device_int4(N: int, K: int, seed: int, dev) -> tuple[torch.Tensor, torch.Tensor]:
    """A seeded fp16 N(0, 0.02^2) matrix generated and quantised on the device
    (the device quantiser is byte-identical to the reference's quantize_w)."""
    from cudalab_b200.int4gemv_quantize import quantize_w_device
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    W = (torch.randn(N, K, generator=g, device=dev) * 0.02).half()
    Wp, s = quantize_w_device(W)
    del W
    return Wp, s


def _x_rows(M: int, K: int, seed: int, dev) -> torch.Tensor:
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return torch.randn(M, K, generator=g, device=dev).half()


def _config4_parity(N, K, world, rank, dev, batches, n_sample=64) -> dict:
    """Fused == NCCL bit for bit, this rank's rows == the single-GPU kernel on
    its shard bit for bit, and sampled rows inside the reference's fixed
    arithmetic bound (int4gemv_correctness.arith_ratio), for every M.  Every
    rank builds the same full matrix; a checksum all-reduce confirms it."""
    from cudalab_b200.build import build
    from cudalab_b200.int4gemv_correctness import arith_ratio
    ext = build("int4gemv")
    Wp, s = _device_int4(N, K, 4242 + N, dev)
    ck = torch.tensor([int(Wp.view(torch.int32).sum().item()) & 0x7fffffff], device=dev,
                      dtype=torch.int64)
    lo, hi = ck.clone(), ck.clone()
    dist.all_reduce(lo, op=dist.ReduceOp.MIN)
    dist.all_reduce(hi, op=dist.ReduceOp.MAX)
    same_w = bool(lo.item() == hi.item())
    row0, n = shard_rows(N, world, rank)
    Ws, ss = Wp[row0:row0 + n].contiguous(), s[row0:row0 + n].contiguous()
    rows = torch.randperm(N, generator=torch.Generator().manual_seed(N + K))[:n_sample]
    Wp_rows, s_rows = Wp[rows.to(dev)].cpu(), s[rows.to(dev)].cpu()
    worst, fused_eq_nccl, shard_eq_single, finite = 0.0, True, True, True
    for M in batches:
        X = _x_rows(M, K, 77 + M, dev)
        xin = X[0] if M == 1 else X
        fused = ShardedGemv("int4gemv", Ws, ss, N, K, mode="fused", max_batch=M)
        nccl = ShardedGemv("int4gemv", Ws, ss, N, K, mode="nccl", max_batch=M)
        try:
            for fl in (0, CONFIG4_FLAGS):
                y_f = fused.forward(xin, flags=fl).clone().view(M, N)
                y_n = nccl.forward(xin, flags=fl).clone().view(M, N)
                y_1 = (ext.forward("int4gemv_mma", Ws, ss, X[0], flags=fl)[None] if M == 1
                       else ext.forward_batched("int4gemv_mma", Ws, ss, X, flags=fl))
                torch.cuda.synchronize(dev)
                fused_eq_nccl &= bool(torch.equal(y_f, y_n))
                shard_eq_single &= bool(torch.equal(y_f[:, row0:row0 + n], y_1))
                finite &= bool(torch.isfinite(y_f.float()).all().item())
                yc, xc = y_f[:, rows.to(dev)].cpu(), X.cpu()
                for m in range(M):
                    r, _, _ = arith_ratio(yc[m], Wp_rows, s_rows, xc[m])
                    worst = max(worst, r)
        finally:
            fused.close()
            torch.cuda.synchronize(dev)
            dist.barrier()
    status = nat.device_status(clear=True)
    ok = torch.tensor([int(same_w and fused_eq_nccl and shard_eq_single and finite
                           and worst <= 1.0 and status == 0)], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    wr = torch.tensor([worst], device=dev, dtype=torch.float64)
    dist.all_reduce(wr, op=dist.ReduceOp.MAX)
    del Wp, s, Ws, ss
    return {"pass": bool(ok.item()), "fused_eq_nccl": fused_eq_nccl,
            "shard_rows_eq_single_gpu": shard_eq_single, "same_weights_all_ranks": same_w,
            "max_arith_ratio_sampled": round(float(wr.item()), 6), "sampled_rows": n_sample}


def config4_block(world: int, rank: int, dev, peak: float, steps: int = 32, reps: int = 10,
                  batches=CONFIG4_BATCHES, modes=("fused", "nccl"), parity: bool = True) -> dict:
    """Time config 4 at this world size and check its parity.  Needs an
    initialised process group (NCCL) of `world` ranks, one GPU each.  Returns
    (on every rank) {"cases": [...], "parity": {...}}; each case has the
    max-over-ranks us per step and the fraction of world x the measured
    per-GPU HBM bandwidth reached on the algorithmic bytes of the full
    matrix."""
    cases = []
    for N, K in CONFIG4_SHAPES:
        row0, n = shard_rows(N, world, rank)
        shard_bytes = n * K // 2 + n * K // 64
        pool = max(2, -(-2 * L2_BYTES // shard_bytes))
        pool += pool % 2
        shards = [_device_int4(n, K, 1000 + 97 * rank + i, dev) for i in range(pool)]
        for M in batches:
            x = _x_rows(M, K, 7, dev)
            x = x[0] if M == 1 else x
            algo = algorithmic_bytes_int4(N, K, M)
            rec = {"shape": f"{N}x{K}", "M": M}
            for mode in modes:
                peers = PeerBuffers(N, max_batch=M) if mode == "fused" else None
                ops = [ShardedGemv("int4gemv", w, s, N, K, mode=mode, peers=peers, max_batch=M)
                       for w, s in shards]
                t, status = time_steps(ops, x, CONFIG4_FLAGS, steps, reps, dev)
                gbs = algo / (t * 1e-6) / 1e9
                rec[mode] = {"us_per_step": round(t, 3),
                             "frac_of_aggregate_hbm": round(gbs / (world * peak), 4),
                             "device_status": status}
                for op in ops:
                    op.close()
                if peers is not None:
                    torch.cuda.synchronize(dev)
                    dist.barrier()
                    peers.close()
            cases.append(rec)
        del shards
        torch.cuda.empty_cache()
    out = {"workload": "int4gemv row-sharded, x replicated, y all-gathered on every rank; "
                       f"pool of weight shards > 2x L2 per rank; flags {CONFIG4_FLAGS}",
           "n_gpus": world, "cases": cases}
    if parity:
        par = {}
        for N, K in CONFIG4_SHAPES:
            par[f"{N}x{K}"] = _config4_parity(N, K, world, rank, dev, batches)
            torch.cuda.empty_cache()
        out["parity"] = par
        out["sharded_parity"] = all(v["pass"] for v in par.values())
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--kinds", default="int4gemv")
    ap.add_argument("--shapes", default="28672x8192,8192x28672")
    ap.add_argument("--modes", default="fused,nccl")
    ap.add_argument("--flags", default="1,3", help="launch flags to time (0, 1=PDL, 3=PDL|inputs ready)")
    ap.add_argument("--batches", default="1", help="activation rows M per step, e.g. 1,4,16")
    ap.add_argument("--steps", type=int, default=32, help="steps per captured graph")
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29541")
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev,
                            rank=rank, world_size=world)
    peak = hbm_peak()
    for kind in a.kinds.split(","):
        for shape in a.shapes.split(","):
            N, K = (int(v) for v in shape.split("x"))
            row0, n = shard_rows(N, world, rank)
            shard_bytes = (n * K // 2 + n * K // 64) if kind == "int4gemv" else (n * K + 4 * n)
            pool = max(2, -(-2 * L2_BYTES // shard_bytes))
            pool += pool % 2
            shards = [make_shard(kind, N, K, row0, n, 1000 + i, dev) for i in range(pool)]
            for M in (int(v) for v in a.batches.split(",")):
                gx = torch.Generator().manual_seed(7)
                x = torch.randn(M, K, generator=gx).half().to(dev)
                x = x[0] if M == 1 else x
                bytes_fn = algorithmic_bytes_int4 if kind == "int4gemv" else algorithmic_bytes_int8
                algo = bytes_fn(N, K, M)
                for mode in a.modes.split(","):
                    peers = PeerBuffers(N, max_batch=M) if mode == "fused" else None
                    ops = [ShardedGemv(kind, w, s, N, K, mode=mode, peers=peers, max_batch=M)
                           for w, s in shards]
                    for fl in (int(f) for f in a.flags.split(",")):
                        t, status = time_steps(ops, x, fl, a.steps, a.reps, dev)
                        gbs = algo / (t * 1e-6) / 1e9
                        if rank == 0:
                            print(json.dumps({
                                "workload": f"sharded {kind} {N}x{K} M={M}", "mode": mode,
                                "flags": fl, "n_gpus": world, "us_per_step": round(t, 3),
                                "gbs_aggregate": round(gbs, 1),
                                "frac_of_aggregate_hbm": round(gbs / (world * peak), 4),
                                "peak_per_gpu_gbs": peak, "pool_per_rank": pool,
                                "rows_per_rank": n, "device_status_max": status}), flush=True)
                    for op in ops:
                        op.close()
                    if peers is not None:
                        torch.cuda.synchronize()
                        dist.barrier()
                        peers.close()
            del shards
            torch.cuda.empty_cache()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
