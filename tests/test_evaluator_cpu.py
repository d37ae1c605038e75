"""Host-side checks of the measurement tools (no GPU needed)."""
import json

import pytest
import torch

from cudalab_b200.evaluator import sweep


def test_sweep_reads_measured_peak():
    peak = sweep.measured_hbm_gbs()
    if (sweep.ROOT / "MEASURED_PEAKS.json").exists():
        data = json.loads((sweep.ROOT / "MEASURED_PEAKS.json").read_text())
        assert peak == pytest.approx(float(data["hbm_gbs"]))
    else:
        assert peak is None


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device refusal")
def test_sweep_refuses_without_a_device():
    with pytest.raises(SystemExit, match="CUDA device"):
        sweep.main(["--kinds", "int4gemv", "--shapes", "256x256"])
