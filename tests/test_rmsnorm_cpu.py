"""RMSNorm oracle pinned by golden vectors the reference itself produced
(cudalab/reference.py rmsnorm_ref on its make_inputs generator, and the fused
RMSNorm -> INT4 layer-A reference; tests/golden/make_golden.py): the oracle
accepts the reference's outputs, its fused bound accepts the reference's
fused outputs, and it rejects outputs moved by two fp16 ulps."""
from pathlib import Path

import numpy as np
import pytest

from oracle import rmsnorm_oracle as orn

G = np.load(Path(__file__).resolve().parent / "golden" / "rmsnorm_golden.npz")
EPS = float(G["eps"])


def _h(b):
    return b.view(np.float16)


CASES = list(range(int(G["n_cases"])))
FUSED = list(range(int(G["n_fused"])))


@pytest.mark.parametrize("i", CASES)
def test_oracle_accepts_reference_rmsnorm(i):
    p = f"c{i}_"
    r = orn.rmsnorm_check(_h(G[p + "y_ref"]), _h(G[p + "x"]), _h(G[p + "w"]), EPS)
    assert r["pass"], r


@pytest.mark.parametrize("i", CASES)
def test_oracle_rejects_two_ulp_moves(i):
    p = f"c{i}_"
    y = _h(G[p + "y_ref"]).copy()
    if not np.any(y):
        pytest.skip("all-zero output")
    k = int(np.argmax(np.abs(y.astype(np.float32))))
    flat = y.reshape(-1)
    flat[k] = np.float16(flat[k].astype(np.float64) + 2 * orn.ulp16(flat[k]))
    assert not orn.rmsnorm_check(y, _h(G[p + "x"]), _h(G[p + "w"]), EPS)["pass"]


@pytest.mark.parametrize("i", FUSED)
def test_fused_bound_accepts_reference(i):
    p = f"f{i}_"
    r = orn.fused_check(_h(G[p + "y_ref"]), G[p + "W_packed"], _h(G[p + "scale"]),
                        _h(G[p + "x"]), _h(G[p + "g"]), EPS)
    assert r["pass"], r
    # the reference's own normalised activations are within one ulp too
    xn = orn.rmsnorm_check(_h(G[p + "xn_ref"]), _h(G[p + "x"]), _h(G[p + "g"]), EPS)
    assert xn["pass"], xn


@pytest.mark.parametrize("i", FUSED)
def test_fused_bound_rejects_moved_output(i):
    p = f"f{i}_"
    y = _h(G[p + "y_ref"]).astype(np.float64)
    y[0, 0] += 0.05 * (np.abs(y).max() + 1.0)
    r = orn.fused_check(y.astype(np.float16), G[p + "W_packed"], _h(G[p + "scale"]),
                        _h(G[p + "x"]), _h(G[p + "g"]), EPS)
    assert not r["pass"], r
