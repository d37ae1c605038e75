"""INT8 parity tests on the GPU: 50-case layer-A suite and 29-case negative
suite per variant, golden vectors, full-size shapes against the oracle."""
from pathlib import Path

import numpy as np
import pytest
import torch

from cudalab_b200 import _native as nat
from cudalab_b200.build import build
from cudalab_b200.operators.qgemv import make_w_q, make_x_q
from cudalab_b200.qgemv_correctness import run_suite, summarize
from cudalab_b200.qgemv_negative import run_negative_suite
from oracle import qgemv_oracle as orc

pytestmark = pytest.mark.gpu
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "qgemv_golden.npz")


@pytest.fixture(scope="module")
def ext():
    return build("qgemv")


def _variants():
    return nat.list_variants("qgemv", nat.CL_VARIANTS_NORMAL)


@pytest.mark.parametrize("variant", _variants())
def test_layer_a_suite(ext, variant):
    res = run_suite(variant, ext)
    s = summarize(res)
    bad = [(r.shape, r.mode, r.arith_max_ratio) for r in res if not r.passed]
    assert s["all_pass"] and s["n_total"] == 50, bad


@pytest.mark.parametrize("variant", _variants())
def test_negative_suite(ext, variant):
    doc = run_negative_suite(ext, variant=variant)
    bad = [(c["id"], c["outcome"], c["first_line"]) for c in doc["cases"] if not c.get("pass")]
    assert doc["summary"]["all_pass"] and doc["summary"]["n_total"] == 29, bad


@pytest.mark.parametrize("variant", _variants())
def test_golden_vectors(ext, variant):
    for i in range(int(GOLD["n_cases"])):
        p = f"c{i}_"
        Wq = torch.from_numpy(GOLD[p + "W_q"]).cuda()
        s = torch.from_numpy(GOLD[p + "scale"]).cuda()
        x = torch.from_numpy(GOLD[p + "x"].view(np.float16).copy()).cuda()
        y = ext.forward(variant, Wq, s, x).cpu().numpy()
        ratio = orc.arith_ratio(y, Wq.shape[1], GOLD[p + "exact"], GOLD[p + "S"])
        assert np.isfinite(y.astype(np.float32)).all()
        assert ratio <= 1.0, (i, ratio)


@pytest.mark.parametrize("shape", [(4096, 4096), (11008, 4096), (4096, 11008), (4096, 1024)],
                         ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("variant", ["qgemv_mma", "qgemv_mma_w4", "qgemv_mma_w8c2", "qgemv_bulk",
                                     "qgemv_ldg"])
def test_full_size_vs_oracle(ext, variant, shape):
    N, K = shape
    Wq, s, _ = make_w_q(N, K, seed=17, scale=0.02)
    x = make_x_q(K, seed=18)
    y = ext.forward(variant, Wq, s, x).cpu().numpy()
    r = orc.check(y, Wq.cpu().numpy(), s.cpu().numpy(), x.cpu().numpy())
    assert r["pass"], r


@pytest.mark.parametrize("variant", _variants())
def test_deterministic_and_pdl_identical(ext, variant):
    Wq, s, _ = make_w_q(2048, 4096, seed=5)
    x = make_x_q(4096, seed=6)
    y0 = ext.forward(variant, Wq, s, x)
    y1 = ext.forward(variant, Wq, s, x)
    y2 = ext.forward(variant, Wq, s, x, flags=nat.CL_LAUNCH_PDL)
    y3 = ext.forward(variant, Wq, s, x, flags=nat.CL_LAUNCH_PDL | nat.CL_LAUNCH_INPUTS_READY)
    assert torch.equal(y0, y1) and torch.equal(y0, y2) and torch.equal(y0, y3)
    assert nat.device_status(clear=True) == 0


@pytest.mark.parametrize("K", [64, 1024, 4096])
@pytest.mark.parametrize("variant", ["qgemv_mma", "qgemv_mma_w4", "qgemv_mma_w8", "qgemv_mma_w8c2",
                                     "qgemv_mma_w16", "qgemv_baseline"])
def test_outlier_rows_vs_oracle(ext, variant, K):
    """Rows with one large weight among tiny ones (quantised values nearly all
    0) and activations spread over six decades."""
    g = torch.Generator().manual_seed(K)
    N = 512
    W = torch.randn(N, K, generator=g) * 1e-3
    W[torch.arange(N), torch.randint(0, K, (N,), generator=g)] = 5.0
    mag = torch.pow(10.0, torch.randint(-3, 3, (K,), generator=g).float())
    x = (torch.randn(K, generator=g) * mag).half()
    from cudalab_b200.qgemv_quantize import quantize_w
    Wq, s = quantize_w(W.half())
    y = ext.forward(variant, Wq.cuda(), s.cuda(), x.cuda()).cpu().numpy()
    r = orc.check(y, Wq.numpy(), s.numpy(), x.numpy())
    assert r["pass"], r
