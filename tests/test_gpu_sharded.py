"""Multi-GPU sharded GEMV (fused peer-store all-gather and NCCL all-gather)
against the single-GPU kernel and the oracle: runs tests/sharded_worker.py
as 2 ranks (and 4 / 8 where the box has that many GPUs) under
torch.distributed.run.  Skipped on a box with one GPU."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_multi_gpu(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs, have {_gpus()}")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
           "--master-port=29533", str(ROOT / "tests" / "sharded_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    out = p.stdout + p.stderr
    assert p.returncode == 0, out[-4000:]
    for r in range(world):
        assert f"SHARDED OK {r}" in out, out[-4000:]
