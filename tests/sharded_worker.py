"""One rank of the multi-GPU sharded-GEMV check (launched by
tests/test_gpu_sharded.py through torch.distributed.run, one process per GPU).

For each case every rank builds the same full weight matrix (CPU generator,
fixed seed), keeps its row shard and runs three steps in fused mode (peer
stores + flags) and in NCCL mode (local GEMV + all-gather), with the launch
flags 0, PDL and PDL|INPUTS_READY.  Checks on every rank:
  * fused y == NCCL y == the single-GPU GEMV of the full matrix, bit for bit
    (the per-row arithmetic does not depend on the sharding);
  * the single-GPU result passes the oracle's bound on sampled rows;
  * no bounded device wait expired.
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
from cudalab_b200.operators.int4gemv import make_w4, make_x4  # noqa: E402
from cudalab_b200.operators.qgemv import make_w_q  # noqa: E402
from cudalab_b200.sharded import ShardedGemv, shard_rows  # noqa: E402
from oracle import int4gemv_oracle as o4  # noqa: E402
from oracle import qgemv_oracle as o8  # noqa: E402

CASES = [("int4gemv", 4096, 4096), ("int4gemv", 1000, 1024), ("qgemv", 4096, 4096),
         ("qgemv", 1000, 1024), ("int4gemv", 28672, 8192), ("int4gemv", 8192, 28672)]


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    nat.device_status(clear=True)
    for kind, N, K in CASES:
        if kind == "int4gemv":
            W, s, _ = make_w4(N, K, seed=N + K, scale=0.02, device="cpu")
            ext = build("int4gemv")
            orc = o4
        else:
            W, s, _ = make_w_q(N, K, seed=N + K, scale=0.02, device="cpu")
            ext = build("qgemv")
            orc = o8
        row0, n = shard_rows(N, world, rank)
        Wd, sd = W.to(dev), s.to(dev)
        fused = ShardedGemv(kind, Wd[row0:row0 + n], sd[row0:row0 + n], N, K, mode="fused")
        nccl = ShardedGemv(kind, Wd[row0:row0 + n], sd[row0:row0 + n], N, K, mode="nccl")
        for step, flags in enumerate((0, nat.CL_LAUNCH_PDL,
                                      nat.CL_LAUNCH_PDL | nat.CL_LAUNCH_INPUTS_READY)):
            x = make_x4(K, seed=100 + step, device="cpu").to(dev)
            y_n = nccl.forward(x, flags=flags).clone()
            y_f = fused.forward(x, flags=flags).clone()
            y_1 = ext.forward("int4gemv_mma" if kind == "int4gemv" else "qgemv_mma", Wd, sd, x,
                              flags=flags)
            torch.cuda.synchronize()
            assert torch.equal(y_f, y_n), (kind, N, K, step, "fused != nccl")
            assert torch.equal(y_f, y_1), (kind, N, K, step, "sharded != single GPU")
            rows = np.random.default_rng(step).choice(N, min(N, 256), replace=False)
            r = orc.check(y_1.cpu().numpy()[rows], W.numpy()[rows], s.numpy()[rows],
                          x.cpu().numpy())
            assert r["pass"], (kind, N, K, step, r)
        st = nat.device_status(clear=True)
        assert st == 0, (kind, N, K, "device status", st)
        fused.close()
        dist.barrier()
    dist.destroy_process_group()
    print(f"SHARDED OK {rank}", flush=True)


if __name__ == "__main__":
    main()
