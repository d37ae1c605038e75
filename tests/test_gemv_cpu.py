"""Dense GEMV on the host: the reference's fixtures (tests/golden/gemv_golden.npz,
made by tests/golden/make_golden.py from the reference's own generators,
gemv_ref and gate) pin the generators, the numpy oracle and the product's
gate restatement; the extension object validates in the reference's order
with its message substrings; the variant lists match the reference's."""
from pathlib import Path

import numpy as np
import pytest
import torch

from cudalab_b200 import gemv_correctness as gc
from cudalab_b200.build import build
from cudalab_b200.operators.gemv import gemv_ref, make_w, make_x
from oracle import gemv_oracle as og

G = np.load(Path(__file__).resolve().parent / "golden" / "gemv_golden.npz")


def _arr(bits: np.ndarray, dt: str) -> np.ndarray:
    return bits.view(np.float16 if dt == "float16" else np.float32)


def _case(i):
    p = f"c{i}_"
    N, K, sw, sx = (int(v) for v in G[p + "meta"])
    dt = str(G[p + "dtype"])
    return dict(N=N, K=K, sw=sw, sx=sx, dt=dt, mode=str(G[p + "mode"]),
                W=_arr(G[p + "W"], dt), x=_arr(G[p + "x"], dt), y_ref=_arr(G[p + "y_ref"], dt),
                exact=G[p + "exact"], S=G[p + "S"], ref_ratio=float(G[p + "ref_ratio"]))


CASES = [_case(i) for i in range(int(G["n_cases"]))]


@pytest.mark.parametrize("c", CASES, ids=lambda c: f"{c['dt']}-{c['N']}x{c['K']}-{c['mode']}")
def test_generators_oracle_gate_against_reference(c):
    dt = getattr(torch, c["dt"])
    W = make_w(c["N"], c["K"], dt, seed=c["sw"], mode=c["mode"], large=10.0)
    x = make_x(c["K"], dt, seed=c["sx"], mode=c["mode"], large=10.0)
    assert W.numpy().tobytes() == c["W"].tobytes()
    assert x.numpy().tobytes() == c["x"].tobytes()
    ex, S = og.exact_and_S(c["W"], c["x"])
    np.testing.assert_allclose(ex, c["exact"], rtol=0, atol=1e-12 * (1 + np.abs(c["exact"]).max()))
    np.testing.assert_allclose(S, c["S"], rtol=1e-15)
    # the product's gate and the oracle's reproduce the reference's ratio of its own result
    y_ref = torch.from_numpy(c["y_ref"].copy())
    r_prod, _, _ = gc.arith_ratio(y_ref, torch.from_numpy(c["W"].copy()),
                                  torch.from_numpy(c["x"].copy()), c["dt"])
    r_orc = og.arith_ratio(c["y_ref"], c["K"], ex, S, c["W"].dtype)
    assert r_prod == pytest.approx(c["ref_ratio"], rel=1e-9, abs=1e-15)
    assert r_orc == pytest.approx(c["ref_ratio"], rel=1e-6, abs=1e-15)  # fp64 sum order
    # the reference's result passes the gate; so does the oracle's fp32 evaluation
    assert og.check(c["y_ref"], c["W"], c["x"])["pass"]
    assert og.check(og.ref_fp32(c["W"], c["x"]), c["W"], c["x"])["pass"]
    assert torch.equal(gemv_ref(torch.from_numpy(c["W"].copy()), torch.from_numpy(c["x"].copy())),
                       y_ref) or c["dt"] == "float32"


def test_gate_catches_a_planted_error():
    c = CASES[0]
    y = c["y_ref"].astype(np.float64).copy()
    y[3] += 0.5  # a gross error on one row
    assert not og.check(y.astype(np.float16), c["W"], c["x"])["pass"]


@pytest.fixture(scope="module")
def ext():
    return build("gemv")


def _rej(fn, sub):
    with pytest.raises(RuntimeError) as ei:
        fn()
    first = str(ei.value).splitlines()[0]
    assert sub in first, first


def test_variant_lists_match_reference(ext):
    assert ext.variants() == ["gemv_baseline", "gemv_mma", "gemv_vec4_row", "gemv_warp_vec4"]
    assert ext.quarantined_variants() == ["gemv_splitk4"]
    assert ext.all_variants() == sorted(ext.variants() + ["gemv_splitk4"])


def test_validation_order_and_messages(ext):
    N, K = 8, 64
    W = torch.zeros(N, K, dtype=torch.float16)
    x = torch.zeros(K, dtype=torch.float16)
    f = lambda a, b: ext.forward("gemv_baseline", a, b)  # noqa: E731
    _rej(lambda: ext.forward("nope", W, x), "未知 gemv 变体")
    _rej(lambda: f(W.view(-1), x), "必须是 2 维")
    _rej(lambda: f(torch.zeros(0, K, dtype=torch.float16), x), "N 必须 > 0")
    _rej(lambda: f(torch.zeros(N, 0, dtype=torch.float16), x), "K 必须 > 0")
    _rej(lambda: f(W.to(torch.bfloat16), x), "float16 / float32")
    _rej(lambda: f(W.to(torch.int32), x), "float16 / float32")
    _rej(lambda: f(torch.zeros(K, N, dtype=torch.float16).t(), x), "连续内存")
    _rej(lambda: f(W, x), "CUDA 张量")  # CPU W: rejected as non-CUDA after the metadata checks
    _rej(lambda: ext.forward_into("gemv_baseline", W, x, torch.zeros(N, dtype=torch.float16)),
         "CUDA 张量")
    _rej(lambda: ext.native_timing("gemv_baseline", W, x, torch.zeros(N), warmup=-1),
         "warmup 必须 >= 0")
