"""Device quantisers (cl_int4gemv_quantize / cl_qgemv_quantize) against the
torch quantisers, which are byte-exact with the reference (tests/golden):
identical W_packed / W_q and scale bytes on every generator mode, on
rounding ties, zero groups / rows and the golden inputs."""
from pathlib import Path

import numpy as np
import pytest
import torch

from cudalab_b200 import int4gemv_quantize as q4
from cudalab_b200 import qgemv_quantize as q8
from cudalab_b200.operators.gemv import make_w as _make_w_fp16

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


def _w(N, K, mode, seed):
    return _make_w_fp16(N, K, torch.float16, device="cpu", seed=seed, mode=mode, scale=1.0,
                        large=10.0)


@pytest.mark.parametrize("mode", ["normal", "zeros", "tiny", "large", "mixed_sign"])
@pytest.mark.parametrize("shape", [(256, 1024), (1000, 4096), (37, 128)], ids=str)
def test_int4_quantize_device_equals_torch(mode, shape):
    W = _w(*shape, mode, seed=shape[0])
    Wp_ref, s_ref = q4.quantize_w(W)
    Wp, s = q4.quantize_w_device(W.cuda())
    assert torch.equal(Wp.cpu(), Wp_ref)
    assert torch.equal(s.cpu().view(torch.int16), s_ref.view(torch.int16))


@pytest.mark.parametrize("mode", ["normal", "zeros", "tiny", "large", "mixed_sign"])
@pytest.mark.parametrize("shape", [(256, 1024), (1000, 4096), (37, 100)], ids=str)
def test_int8_quantize_device_equals_torch(mode, shape):
    W = _w(*shape, mode, seed=shape[0])
    Wq_ref, s_ref = q8.quantize_w(W)
    Wq, s = q8.quantize_w_device(W.cuda())
    assert torch.equal(Wq.cpu(), Wq_ref)
    assert torch.equal(s.cpu().view(torch.int32), s_ref.view(torch.int32))


def test_quantize_ties_and_zero_groups():
    """Values exactly halfway between two quantisation steps (round half to
    even), a group of zeros and a group with one non-zero element."""
    K = 256
    W = torch.zeros(4, K, dtype=torch.float16)
    W[0, :128] = 7.0
    W[0, 1:128:2] = torch.tensor([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5] * 8)
    W[1, 130] = -3.0
    W[2] = torch.linspace(-14, 14, K).half()
    for fn in ((q4.quantize_w, q4.quantize_w_device), (q8.quantize_w, q8.quantize_w_device)):
        a = fn[0](W)
        b = fn[1](W.cuda())
        for x, y in zip(a, b):
            assert torch.equal(x.view(torch.uint8), y.cpu().view(torch.uint8))


def test_quantize_golden_inputs():
    g = np.load(GOLD / "int4gemv_golden.npz")
    for i in range(int(g["n_cases"])):
        W = torch.from_numpy(g[f"c{i}_W_fp16"].view(np.float16).copy())
        Wp, s = q4.quantize_w_device(W.cuda())
        assert np.array_equal(Wp.cpu().numpy(), g[f"c{i}_W_packed"])
        assert np.array_equal(s.cpu().numpy().view(np.uint16), g[f"c{i}_scale"].view(np.uint16))


def test_quantize_rejects():
    with pytest.raises(ValueError):
        q4.quantize_w_device(torch.zeros(4, 100, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):
        q4.quantize_w_device(torch.full((4, 128), float("inf"), dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):
        q8.quantize_w_device(torch.zeros(4, 128, dtype=torch.float32, device="cuda"))
