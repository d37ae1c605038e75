"""Batched activations (X [M, K] -> Y [M, N]) through the C ABI on the GPU.

Every output row is checked against the oracle's fixed bound (the reference's
arithmetic gate applied per activation row); M = 1 through the batched entry
point must equal the single-vector entry point bit for bit.  Shapes cover the
K-split clusters (few row tiles, or staged activations too large for one CTA),
several rounds of the partial buffer, partial last chunks and ragged N."""
import numpy as np
import pytest
import torch

from cudalab_b200 import _native as nat
from cudalab_b200.build import build
from cudalab_b200.operators.int4gemv import make_w4
from cudalab_b200.operators.qgemv import make_w_q
from oracle import int4gemv_oracle as o4
from oracle import qgemv_oracle as o8

pytestmark = pytest.mark.gpu

MMA4 = ["int4gemv_mma", "int4gemv_mma_w4", "int4gemv_mma_w8", "int4gemv_mma_w8c2",
        "int4gemv_mma_w16"]
MMA8 = [v.replace("int4gemv", "qgemv") for v in MMA4]
# the 5th-generation tensor-core kernel (tcgen05, TMEM, TMA); INT4 only
TC4 = ["int4gemv_tc"]


def _x(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(M, K, generator=g).half()


def _check_rows(orc, Y, W, s, X, rows=None):
    Wn, sn = W.cpu().numpy(), s.cpu().numpy()
    if rows is not None:
        Wn, sn, Y = Wn[rows], sn[rows], Y[:, rows]
    for m in range(X.shape[0]):
        r = orc.check(Y[m], Wn, sn, X[m])
        assert r["pass"], (m, r)


# (N, K, M): plain, ragged N, K-split by few tiles, partial chunks, rounds
SHAPES4 = [(4096, 4096, 4), (1000, 1024, 3), (256, 8192, 16), (4096, 1152, 9),
           (16384, 8192, 16), (1024, 28672, 16), (4096, 4096, 17)]


@pytest.mark.parametrize("shape", SHAPES4, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("variant", MMA4 + TC4)
def test_int4_batched_vs_oracle(variant, shape):
    N, K, M = shape
    ext = build("int4gemv")
    W, s, _ = make_w4(N, K, seed=N + K, scale=0.02)
    X = _x(M, K, seed=M)
    Y = ext.forward_batched(variant, W, s, X.cuda()).cpu().numpy()
    rows = None if N * K <= 4096 * 4096 else np.random.default_rng(0).choice(N, 512, replace=False)
    _check_rows(o4, Y, W, s, X.numpy(), rows)
    assert nat.device_status(clear=True) == 0


SHAPES8 = [(4096, 4096, 4), (1000, 1024, 3), (256, 8192, 16), (4096, 1088, 9),
           (1024, 28672, 16)]


@pytest.mark.parametrize("shape", SHAPES8, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("variant", MMA8)
def test_int8_batched_vs_oracle(variant, shape):
    N, K, M = shape
    ext = build("qgemv")
    W, s, _ = make_w_q(N, K, seed=N + K, scale=0.02)
    X = _x(M, K, seed=M)
    Y = ext.forward_batched(variant, W, s, X.cuda()).cpu().numpy()
    _check_rows(o8, Y, W, s, X.numpy())
    assert nat.device_status(clear=True) == 0


@pytest.mark.parametrize("variant", ["int4gemv_mma", "int4gemv_bulk", "int4gemv_baseline"])
def test_batched_m1_equals_single(variant):
    ext = build("int4gemv")
    W, s, _ = make_w4(2048, 4096, seed=1)
    X = _x(1, 4096, seed=2).cuda()
    assert torch.equal(ext.forward_batched(variant, W, s, X)[0], ext.forward(variant, W, s, X[0]))


@pytest.mark.parametrize("variant", ["int4gemv_bulk", "int4gemv_baseline"])
def test_batched_per_row_variants(variant):
    """Variants without a batch dimension run once per row: row m equals the
    single-vector call on X[m] bit for bit."""
    ext = build("int4gemv")
    W, s, _ = make_w4(1024, 2048, seed=3)
    X = _x(5, 2048, seed=4).cuda()
    Y = ext.forward_batched(variant, W, s, X)
    for m in range(5):
        assert torch.equal(Y[m], ext.forward(variant, W, s, X[m]))


@pytest.mark.parametrize("flags", [0, 1, 3])
def test_batched_flags_identical(flags):
    ext = build("int4gemv")
    W, s, _ = make_w4(4096, 4096, seed=5)
    X = _x(8, 4096, seed=6).cuda()
    ref = ext.forward_batched("int4gemv_mma", W, s, X)
    assert torch.equal(ext.forward_batched("int4gemv_mma", W, s, X, flags=flags), ref)


@pytest.mark.parametrize("flags", [0, 1, 3])
@pytest.mark.parametrize("shape", [(1024, 4096), (256, 8192), (4096, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
def test_single_vector_flags_identical_across_geometry(shape, flags):
    """The K split (summation order) depends on the shape only, so the auto
    variant gives the same bits whatever geometry the launch flags select."""
    N, K = shape
    ext = build("int4gemv")
    W, s, _ = make_w4(N, K, seed=7)
    x = _x(1, K, seed=8)[0].cuda()
    ref = ext.forward("int4gemv_mma_w8", W, s, x)
    assert torch.equal(ext.forward("int4gemv_mma", W, s, x, flags=flags), ref)


def test_batched_rejects():
    ext = build("int4gemv")
    W, s, _ = make_w4(256, 1024, seed=9)
    for bad in (torch.zeros(0, 1024, dtype=torch.float16, device="cuda"),
                torch.zeros(2, 512, dtype=torch.float16, device="cuda"),
                torch.zeros(2, 1024, dtype=torch.float32, device="cuda"),
                torch.zeros(1024, dtype=torch.float16, device="cuda")):
        with pytest.raises(RuntimeError):
            ext.forward_batched("int4gemv_mma", W, s, bad)


@pytest.mark.parametrize("flags", [0, 1, 3, 7])
@pytest.mark.parametrize("M", [1, 16])
def test_tc_flags_identical(flags, M):
    """Launch flags change scheduling only: the tcgen05 kernel's K split (and
    summation order) depends on the shape and the SM count."""
    ext = build("int4gemv")
    W, s, _ = make_w4(1024, 8192, seed=11)
    X = _x(M, 8192, seed=12).cuda()
    ref = ext.forward_batched("int4gemv_tc", W, s, X)
    assert torch.equal(ext.forward_batched("int4gemv_tc", W, s, X, flags=flags), ref)
    assert nat.device_status(clear=True) == 0


def test_tc_misaligned_scales_and_zero_rows():
    """Scale rows at an odd half offset, a zero weight matrix and zero
    activation rows: the tcgen05 kernel reads scales one at a time and its
    results stay inside the bound (zeros exactly)."""
    ext = build("int4gemv")
    W, s, _ = make_w4(640, 2048, seed=13)
    buf = torch.empty(s.numel() + 1, dtype=torch.float16, device="cuda")
    s2 = buf[1:].view(s.shape)
    s2.copy_(s)
    X = _x(5, 2048, seed=14)
    X[2].zero_()
    Y = ext.forward_batched("int4gemv_tc", W, s2, X.cuda()).cpu().numpy()
    _check_rows(o4, Y, W, s, X.numpy())
    assert not Y[2].any()
    Z = ext.forward_batched("int4gemv_tc", torch.zeros_like(W), s, X.cuda())
    assert not Z.any()
    assert nat.device_status(clear=True) == 0
