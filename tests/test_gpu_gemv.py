"""Dense GEMV (fp16 / fp32) on the GPU through the C ABI:

  * the 100-case correctness suite (2 dtypes x 10 shapes x 5 modes) per variant;
  * the 24-case negative suite per variant (including the quarantined
    gemv_splitk4, run by explicit name as the reference allows);
  * the reference's golden vectors on every variant;
  * determinism and launch-flag independence of the tensor-core fp16 path,
    its baseline fallback (bits), full-size shapes, native timing.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from cudalab_b200 import _native as nat
from cudalab_b200.build import build
from cudalab_b200.gemv_correctness import run_suite, summarize
from cudalab_b200.gemv_negative import run_negative_suite
from cudalab_b200.operators.gemv import make_w, make_x
from oracle import gemv_oracle as orc

pytestmark = pytest.mark.gpu
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "gemv_golden.npz")
ALL = ["gemv_baseline", "gemv_mma", "gemv_splitk4", "gemv_vec4_row", "gemv_warp_vec4"]


@pytest.fixture(scope="module")
def ext():
    return build("gemv")


@pytest.mark.parametrize("variant", ALL)
def test_correctness_suite(ext, variant):
    res = run_suite(variant, ext)
    s = summarize(res)
    bad = [(r.dtype, r.shape, r.mode, r.arith_max_ratio) for r in res if not r.passed]
    assert s["n_total"] == 100 and s["all_pass"], bad


@pytest.mark.parametrize("variant", ALL)
def test_negative_suite(ext, variant):
    doc = run_negative_suite(ext, variant=variant)
    bad = [(c["id"], c["outcome"], c["first_line"]) for c in doc["cases"] if not c.get("pass")]
    assert doc["summary"]["all_pass"] and doc["summary"]["n_total"] == 24, bad


@pytest.mark.parametrize("variant", ALL)
def test_golden_vectors(ext, variant):
    for i in range(int(GOLD["n_cases"])):
        p = f"c{i}_"
        dt = str(GOLD[p + "dtype"])
        npdt = np.float16 if dt == "float16" else np.float32
        W = torch.from_numpy(GOLD[p + "W"].view(npdt).copy()).cuda()
        x = torch.from_numpy(GOLD[p + "x"].view(npdt).copy()).cuda()
        y = ext.forward(variant, W, x).cpu().numpy()
        ratio = orc.arith_ratio(y, W.shape[1], GOLD[p + "exact"], GOLD[p + "S"], npdt)
        assert np.isfinite(y.astype(np.float64)).all()
        assert ratio <= 1.0, (i, dt, ratio)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32], ids=["f16", "f32"])
@pytest.mark.parametrize("shape", [(4096, 4096), (11008, 4096), (4096, 11008), (28672, 8192)],
                         ids=lambda s: f"{s[0]}x{s[1]}")
def test_full_size_vs_oracle(ext, shape, dtype):
    N, K = shape
    W = make_w(N, K, dtype, device="cuda", seed=31, scale=0.02)
    x = make_x(K, dtype, device="cuda", seed=32)
    for v in ("gemv_mma", "gemv_warp_vec4"):
        y = ext.forward(v, W, x).cpu().numpy()
        rows = np.random.default_rng(0).choice(N, size=min(N, 512), replace=False)
        r = orc.check(y[rows], W.cpu().numpy()[rows], x.cpu().numpy())
        assert r["pass"], (v, r)


def test_mma_deterministic_and_flags_identical(ext):
    W = make_w(3000, 4096, torch.float16, device="cuda", seed=5)
    x = make_x(4096, torch.float16, device="cuda", seed=6)
    ys = [ext.forward("gemv_mma", W, x, flags=f) for f in (0, 0, 1, 3, 7)]
    assert all(torch.equal(ys[0], y) for y in ys[1:])
    assert nat.device_status(clear=True) == 0


@pytest.mark.parametrize("K", [40, 4104, 13])
def test_mma_fallback_is_baseline_bits(ext, K):
    # K not a multiple of 32: the tensor-core path runs the baseline kernel
    W = make_w(257, K, torch.float16, device="cuda", seed=K)
    x = make_x(K, torch.float16, device="cuda", seed=K + 1)
    assert torch.equal(ext.forward("gemv_mma", W, x), ext.forward("gemv_baseline", W, x))


@pytest.mark.parametrize("K", [32, 96, 4128])
def test_mma_ragged_rows_vs_oracle(ext, K):
    # K a multiple of 32 but not of 128: a short last chunk per row
    W = make_w(777, K, torch.float16, device="cuda", seed=K, mode="mixed_sign")
    x = make_x(K, torch.float16, device="cuda", seed=K + 1, mode="mixed_sign")
    y = ext.forward("gemv_mma", W, x).cpu().numpy()
    assert orc.check(y, W.cpu().numpy(), x.cpu().numpy())["pass"]


def test_native_timing(ext):
    W = make_w(4096, 4096, torch.float16, device="cuda", seed=1)
    x = make_x(4096, torch.float16, device="cuda", seed=2)
    out = torch.empty(4096, dtype=torch.float16, device="cuda")
    d = ext.native_timing("gemv_mma", W, x, out, warmup=5, n_windows=3, launches_per_window=8)
    assert d["variant"] == "gemv_mma" and len(d["window_median_us"]) == 3
    assert 0 < d["min_us"] <= d["median_us"] <= d["max_us"]
