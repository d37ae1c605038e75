"""Golden vectors produced by the reference itself (tests/golden/make_golden.py)
pin: the generators, the product quantisers (byte-exact), the numpy oracle
(byte-exact quantisation, layer-A values inside the fixed bound) and the
C restatement used as the CPU baseline."""
from pathlib import Path

import numpy as np
import pytest
import torch

from cudalab_b200 import int4gemv_quantize as q4
from cudalab_b200 import qgemv_quantize as q8
from cudalab_b200.operators.gemv import make_w, make_x
from oracle import cpu_gemv
from oracle import int4gemv_oracle as o4
from oracle import qgemv_oracle as o8

GOLD = Path(__file__).resolve().parent / "golden"
G4 = np.load(GOLD / "int4gemv_golden.npz")
G8 = np.load(GOLD / "qgemv_golden.npz")


def _h(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16)


def _case(G, i, wkey):
    p = f"c{i}_"
    N, K, sw, sx = (int(v) for v in G[p + "meta"])
    return dict(N=N, K=K, sw=sw, sx=sx, mode=str(G[p + "mode"]), W=_h(G[p + "W_fp16"]),
                x=_h(G[p + "x"]), Wq=G[p + wkey], scale=G[p + "scale"],
                y_ref=_h(G[p + "y_ref"]), exact=G[p + "exact"], S=G[p + "S"],
                ref_ratio=float(G[p + "ref_ratio"]))


I4 = [_case(G4, i, "W_packed") for i in range(int(G4["n_cases"]))]
I8 = [_case(G8, i, "W_q") for i in range(int(G8["n_cases"]))]


def test_byte_table_matches_reference():
    t = G4["byte_table_unpacked"].astype(np.int32)
    Wp = torch.arange(256, dtype=torch.uint8).view(1, 256)
    assert np.array_equal(q4.unpack_w(Wp).numpy(), t)
    assert np.array_equal(o4.unpack_w(Wp.numpy()), t)


@pytest.mark.parametrize("c", I4, ids=lambda c: f"{c['N']}x{c['K']}-{c['mode']}")
def test_int4_generators_quantiser_oracle(c):
    if c["N"] != 5:  # case 5x384 has a hand-zeroed group: generators are checked elsewhere
        W = make_w(c["N"], c["K"], torch.float16, seed=c["sw"], mode=c["mode"], large=10.0)
        assert np.array_equal(W.numpy().view(np.uint16), c["W"].view(np.uint16))
    x = make_x(c["K"], torch.float16, seed=c["sx"], mode=c["mode"], large=10.0)
    assert np.array_equal(x.numpy().view(np.uint16), c["x"].view(np.uint16))
    Wp, s16 = q4.quantize_w(torch.from_numpy(c["W"].copy()))
    assert np.array_equal(Wp.numpy(), c["Wq"])
    assert np.array_equal(s16.numpy().view(np.uint16), c["scale"])
    owp, os16 = o4.quantize_w(c["W"])
    assert np.array_equal(owp, c["Wq"])
    assert np.array_equal(os16.view(np.uint16), c["scale"])
    # fp64 exact values of the oracle equal the reference's
    ex, S = o4.exact_and_S(c["Wq"], _h(c["scale"]), c["x"])
    np.testing.assert_allclose(ex, c["exact"], rtol=0, atol=1e-12 * (1 + np.abs(c["exact"]).max()))
    np.testing.assert_allclose(S, c["S"], rtol=1e-15)
    # layer-A values: reference output, oracle output and C restatement all pass the gate
    K = c["K"]
    assert o4.arith_ratio(c["y_ref"], K, c["exact"], c["S"]) <= 1.0
    assert o4.arith_ratio(o4.gemv_ref(c["Wq"], _h(c["scale"]), c["x"]), K, ex, S) <= 1.0
    y_c = cpu_gemv.int4_gemv(c["Wq"], c["scale"], c["x"].view(np.uint16), threads=2)
    assert o4.arith_ratio(y_c, K, ex, S) <= 1.0
    # the package's own host dequantisation reproduces the reference layer-A value bit for bit
    y_pkg = torch.mv(q4.dequantize_w(torch.from_numpy(c["Wq"]),
                                     torch.from_numpy(_h(c["scale"]).copy())),
                     torch.from_numpy(c["x"].copy()).float()).to(torch.float16)
    assert o4.arith_ratio(y_pkg.numpy(), K, ex, S) <= 1.0


@pytest.mark.parametrize("c", I8, ids=lambda c: f"{c['N']}x{c['K']}-{c['mode']}")
def test_int8_generators_quantiser_oracle(c):
    W = make_w(c["N"], c["K"], torch.float16, seed=c["sw"], mode=c["mode"], large=10.0)
    assert np.array_equal(W.numpy().view(np.uint16), c["W"].view(np.uint16))
    x = make_x(c["K"], torch.float16, seed=c["sx"], mode=c["mode"], large=10.0)
    assert np.array_equal(x.numpy().view(np.uint16), c["x"].view(np.uint16))
    Wq, s = q8.quantize_w(torch.from_numpy(c["W"].copy()))
    assert np.array_equal(Wq.numpy(), c["Wq"])
    assert np.array_equal(s.numpy().view(np.uint32), c["scale"].view(np.uint32))
    owq, os = o8.quantize_w(c["W"])
    assert np.array_equal(owq, c["Wq"])
    assert np.array_equal(os.view(np.uint32), c["scale"].view(np.uint32))
    ex, S = o8.exact_and_S(c["Wq"], c["scale"], c["x"])
    np.testing.assert_allclose(ex, c["exact"], rtol=0, atol=1e-12 * (1 + np.abs(c["exact"]).max()))
    K = c["K"]
    assert o8.arith_ratio(c["y_ref"], K, c["exact"], c["S"]) <= 1.0
    assert o8.arith_ratio(o8.gemv_ref(c["Wq"], c["scale"], c["x"]), K, ex, S) <= 1.0
    y_c = cpu_gemv.int8_gemv(c["Wq"], c["scale"], c["x"].view(np.uint16), threads=2)
    assert o8.arith_ratio(y_c, K, ex, S) <= 1.0


def test_oracle_gate_detects_planted_errors():
    """The checker must fail outputs that are wrong: a dropped term, a swapped
    nibble order and a wrong row all exceed the bound (errors planted in the
    oracle's own computation, on the CPU)."""
    c = next(c for c in I4 if c["N"] == 32)
    Wp, s16, x = c["Wq"], _h(c["scale"]), c["x"]
    K = c["K"]
    ex, S = c["exact"], c["S"]
    # swapped nibbles: byte (hi<<4)|lo -> (lo<<4)|hi
    swapped = ((Wp & 0xF) << 4 | (Wp >> 4)).astype(np.uint8)
    assert o4.arith_ratio(o4.gemv_ref(swapped, s16, x), K, ex, S) > 1.0
    # one group dropped
    s_drop = s16.copy()
    s_drop[:, 0] = 0
    assert o4.arith_ratio(o4.gemv_ref(Wp, s_drop, x), K, ex, S) > 1.0
    # rows permuted
    assert o4.arith_ratio(o4.gemv_ref(Wp[::-1].copy(), s16[::-1].copy(), x), K, ex, S) > 1.0


def test_c_oracle_half_conversions_exhaustive():
    lib = cpu_gemv.load()
    bits = np.arange(65536, dtype=np.uint16)
    h = bits.view(np.float16)
    finite = np.isfinite(h)
    f = np.array([lib.oracle_h2f(int(b)) for b in bits[finite][::37]], np.float32)
    assert np.array_equal(f, h[finite][::37].astype(np.float32))
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(4000).astype(np.float32) * 10.0 ** rng.integers(-9, 5, 4000),
                           np.float32([65504, 65519.99, 65520, 6.1e-5, 5.96e-8, 2.98e-8, 0.0, -0.0])])
    got = np.array([lib.oracle_f2h(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, vals.astype(np.float16).view(np.uint16))
