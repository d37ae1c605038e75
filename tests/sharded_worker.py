"""One rank of the multi-GPU sharded-GEMV check (launched by
tests/test_gpu_sharded.py through torch.distributed.run, one process per GPU).

For each case every rank builds the same full weight matrix (CPU generator,
fixed seed), keeps its row shard and runs three steps in fused mode (peer
stores + flags) and in NCCL mode (local GEMV + all-gather), with the launch
flags 0, PDL and PDL|INPUTS_READY.  Checks on every rank:
  * fused y == NCCL y bit for bit, and this rank's rows == the single-GPU
    GEMV of its shard bit for bit (same kernel, same geometry);
  * y passes the oracle's bound on sampled rows;
  * no bounded device wait expired.
Batched cases (M > 1) run the same checks per activation row.
Prints "SHARDED OK <rank>" on success.
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from cudalab_b200 import _native as nat  # noqa: E402
from cudalab_b200.build import build  # noqa: E402
from cudalab_b200.operators.int4gemv import make_w4  # noqa: E402
from cudalab_b200.operators.qgemv import make_w_q  # noqa: E402
from cudalab_b200.sharded import ShardedGemv, shard_rows  # noqa: E402
from oracle import int4gemv_oracle as o4  # noqa: E402
from oracle import qgemv_oracle as o8  # noqa: E402

CASES = [("int4gemv", 4096, 4096, 1), ("int4gemv", 1000, 1024, 1), ("qgemv", 4096, 4096, 1),
         ("qgemv", 1000, 1024, 1), ("int4gemv", 28672, 8192, 1), ("int4gemv", 8192, 28672, 1),
         ("int4gemv", 4096, 4096, 4), ("int4gemv", 8192, 28672, 16), ("qgemv", 4096, 4096, 16)]


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    nat.device_status(clear=True)
    for kind, N, K, M in CASES:
        if kind == "int4gemv":
            W, s, _ = make_w4(N, K, seed=N + K, scale=0.02, device="cpu")
            ext = build("int4gemv")
            orc = o4
        else:
            W, s, _ = make_w_q(N, K, seed=N + K, scale=0.02, device="cpu")
            ext = build("qgemv")
            orc = o8
        row0, n = shard_rows(N, world, rank)
        Wd, sd = W[row0:row0 + n].contiguous().to(dev), s[row0:row0 + n].contiguous().to(dev)
        fused = ShardedGemv(kind, Wd, sd, N, K, mode="fused", max_batch=M)
        nccl = ShardedGemv(kind, Wd, sd, N, K, mode="nccl", max_batch=M)
        variant = "int4gemv_mma" if kind == "int4gemv" else "qgemv_mma"
        for step, flags in enumerate((0, nat.CL_LAUNCH_PDL,
                                      nat.CL_LAUNCH_PDL | nat.CL_LAUNCH_INPUTS_READY)):
            g = torch.Generator().manual_seed(100 + step)
            X = torch.randn(M, K, generator=g).half().to(dev)
            xin = X[0] if M == 1 else X
            y_n = nccl.forward(xin, flags=flags).clone()
            y_f = fused.forward(xin, flags=flags).clone()
            if M == 1:
                y_1 = ext.forward(variant, Wd, sd, X[0], flags=flags)[None]
                y_f2, y_n2 = y_f[None], y_n[None]
            else:
                y_1 = ext.forward_batched(variant, Wd, sd, X, flags=flags)
                y_f2, y_n2 = y_f, y_n
            torch.cuda.synchronize()
            assert torch.equal(y_f2, y_n2), (kind, N, K, M, step, "fused != nccl")
            assert torch.equal(y_f2[:, row0:row0 + n], y_1), (kind, N, K, M, step, "shard rows")
            rows = np.random.default_rng(step).choice(N, min(N, 256), replace=False)
            Yc, Xc = y_f2.cpu().numpy(), X.cpu().numpy()
            for m in range(M):
                r = orc.check(Yc[m][rows], W.numpy()[rows], s.numpy()[rows], Xc[m])
                assert r["pass"], (kind, N, K, M, m, step, r)
        st = nat.device_status(clear=True)
        assert st == 0, (kind, N, K, M, "device status", st)
        fused.close()
        dist.barrier()
    dist.destroy_process_group()
    print(f"SHARDED OK {rank}", flush=True)


if __name__ == "__main__":
    main()
