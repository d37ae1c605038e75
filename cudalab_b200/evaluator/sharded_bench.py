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
