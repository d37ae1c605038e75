"""bench.py's reference arm on the CPU: one JSON line with the contract's keys,
the same metric, unit, direction and config as the GPU arm reports (the
config comes from one function both arms call), and a bounded sample."""
import json
import subprocess
import sys
from argparse import Namespace
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402

LIB = ROOT / "oracle" / "_build" / "libcpu_gemv.so"


@pytest.mark.skipif(not LIB.exists(), reason="oracle/_build not built (make -C oracle)")
def test_reference_arm_line_matches_gpu_arm_contract():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "3"], cwd=ROOT, capture_output=True,
                         text=True, timeout=300, check=True).stdout.strip().splitlines()
    line = json.loads(out[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "GB/s"
    assert line["higher_is_better"] is True
    assert line["config"] == bench.arm_config(Namespace(mode="independent"), 1)
    assert line["steps"] == 1 and line["warmup"] == 3 and line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert "rows of one 4096x4096 weight set" in cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
