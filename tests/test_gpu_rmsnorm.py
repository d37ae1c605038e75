"""RMSNorm and the fused RMSNorm -> INT4 GEMV on the GPU, through the C ABI.

* cl_rmsnorm_f16 on the reference's own inputs (golden fixtures made by its
  make_inputs / rmsnorm_ref): every element within one fp16 ulp of the
  correctly rounded fp64 value (the oracle's gate, which also accepts the
  reference's outputs).
* cl_int4gemv_rmsnorm on the golden fused cases: within the INT4 arithmetic
  bound widened by one fp16 ulp per normalised activation.
* At every size, including the headline shapes: the fused launch equals
  cl_rmsnorm_f16 followed by the batched GEMV (variant int4gemv_mma_w8c2)
  bit for bit, for every fused variant, M from 1 to 20 and both launch modes
  (a size-independent property: the normalised activations never leave the
  CTA, so this is the check that they are the standalone kernel's bits).
* The contract: misaligned norm weight, negative / non-finite eps, K not a
  multiple of 128 are rejected before any launch or by the launch itself."""
from pathlib import Path

import numpy as np
import pytest
import torch

from cudalab_b200 import _native as nat
from cudalab_b200.build import build
from cudalab_b200.operators.int4gemv import make_w4
from oracle import rmsnorm_oracle as orn

pytestmark = pytest.mark.gpu

G = np.load(Path(__file__).resolve().parent / "golden" / "rmsnorm_golden.npz")
EPS = float(G["eps"])
FUSED_VARIANTS = ["int4gemv_rmsnorm", "int4gemv_rmsnorm_w2", "int4gemv_rmsnorm_w4",
                  "int4gemv_rmsnorm_w8", "int4gemv_rmsnorm_w8c2", "int4gemv_rmsnorm_w16"]


def _h(b):
    return torch.from_numpy(b.view(np.float16).copy())


def _rows(M, K, seed, mode="normal"):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    if mode == "biased":
        x = x + 3.0
    elif mode == "tiny":
        x = x * 1e-4
    w = torch.randn(K, generator=g) * 0.5 + 1.0
    return x.half(), w.half()


@pytest.mark.parametrize("i", range(int(G["n_cases"])))
def test_rmsnorm_vs_golden(i):
    ext = build("rmsnorm")
    p = f"c{i}_"
    M, H, _ = (int(v) for v in G[p + "meta"])
    x, w = _h(G[p + "x"]).view(M, H), _h(G[p + "w"])
    y = ext.forward("rmsnorm_f16", x.cuda(), w.cuda(), EPS).cpu()
    r = orn.rmsnorm_check(y.numpy(), x.numpy(), w.numpy(), EPS)
    assert r["pass"], r
    # against the reference's own output: the same gate holds for both
    ref = G[p + "y_ref"].view(np.float16).reshape(M, H)
    assert orn.rmsnorm_check(ref, x.numpy(), w.numpy(), EPS)["pass"]


@pytest.mark.parametrize("shape", [(1, 8), (5, 4096), (3, 8192), (2, 24576), (7, 1000)])
@pytest.mark.parametrize("mode", ["normal", "biased", "tiny"])
def test_rmsnorm_random_vs_oracle(shape, mode):
    ext = build("rmsnorm")
    M, H = shape
    x, w = _rows(M, H, seed=M * H, mode=mode)
    y = ext.forward("rmsnorm_f16", x.cuda(), w.cuda()).cpu()
    r = orn.rmsnorm_check(y.numpy(), x.numpy(), w.numpy(), EPS)
    assert r["pass"], r


def test_rmsnorm_zero_rows():
    ext = build("rmsnorm")
    x = torch.zeros(2, 512, dtype=torch.float16, device="cuda")
    w = torch.ones(512, dtype=torch.float16, device="cuda")
    assert torch.count_nonzero(ext.forward("rmsnorm_f16", x, w)).item() == 0


@pytest.mark.parametrize("i", range(int(G["n_fused"])))
@pytest.mark.parametrize("variant", FUSED_VARIANTS)
def test_fused_vs_golden(variant, i):
    ext = build("int4gemv")
    p = f"f{i}_"
    N, K, M, _, _ = (int(v) for v in G[p + "meta"])
    Wp = torch.from_numpy(G[p + "W_packed"].copy())
    s = _h(G[p + "scale"]).view(N, K // 128)
    x, g = _h(G[p + "x"]).view(M, K), _h(G[p + "g"])
    y = ext.forward_rmsnorm(variant, Wp.cuda(), s.cuda(), x.cuda(), g.cuda(), EPS).cpu()
    r = orn.fused_check(y.numpy(), Wp.numpy(), s.numpy(), x.numpy(), g.numpy(), EPS)
    assert r["pass"], r
    assert nat.device_status(clear=True) == 0


def _separate(W, s, X, g, eps, flags=0):
    """RMSNorm, then the batched GEMV with the same geometry: the unfused path."""
    xn = build("rmsnorm").forward("rmsnorm_f16", X, g, eps, flags=flags)
    return build("int4gemv").forward_batched("int4gemv_mma_w8c2", W, s, xn, flags=flags)


# (N, K, M): small, ragged N, K split across a cluster (few row tiles), the
# decoder projections at full size, more than 16 rows (two launches)
SHAPES = [(256, 1024, 1), (1000, 2048, 3), (256, 8192, 16), (4096, 4096, 1), (4096, 4096, 8),
          (28672, 8192, 1), (8192, 28672, 4), (4096, 4096, 20), (14336, 4096, 9)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_fused_equals_separate(shape):
    N, K, M = shape
    ext = build("int4gemv")
    W, s, _ = make_w4(N, K, seed=N + K, scale=0.02)
    X, g = _rows(M, K, seed=M + K)
    X, g = X.cuda(), g.cuda()
    ref = _separate(W, s, X, g, EPS)
    for variant in FUSED_VARIANTS:
        for flags in (0, 3):
            y = ext.forward_rmsnorm(variant, W, s, X, g, EPS, flags=flags)
            torch.cuda.synchronize()
            assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), (variant, flags)
    assert nat.device_status(clear=True) == 0


def test_fused_one_dim_and_out():
    ext = build("int4gemv")
    N, K = 512, 2048
    W, s, _ = make_w4(N, K, seed=3, scale=0.02)
    X, g = _rows(1, K, seed=5)
    X, g = X.cuda(), g.cuda()
    y2 = ext.forward_rmsnorm("int4gemv_rmsnorm", W, s, X, g)
    y1 = ext.forward_rmsnorm("int4gemv_rmsnorm", W, s, X[0], g)
    assert y1.shape == (N,) and torch.equal(y1, y2[0])
    out = torch.empty(1, N, dtype=torch.float16, device="cuda")
    ext.forward_rmsnorm("int4gemv_rmsnorm", W, s, X, g, out=out)
    assert torch.equal(out, y2)


def test_fused_misaligned_scale_and_ragged_rows():
    # scale rows not 8-byte aligned (the general fetch path) and N not a
    # multiple of the 16-row tile
    ext = build("int4gemv")
    N, K = 77, 384
    W, s, _ = make_w4(N, K, seed=9, scale=0.02)
    buf = torch.empty(N * 3 + 1, dtype=torch.float16, device="cuda")
    s_odd = buf[1:].view(N, 3)
    s_odd.copy_(s)
    X, g = _rows(3, K, seed=11, mode="biased")
    X, g = X.cuda(), g.cuda()
    ref = _separate(W, s, X, g, EPS)
    for variant in FUSED_VARIANTS:
        y = ext.forward_rmsnorm(variant, W, s_odd, X, g, EPS)
        assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), variant


def test_fused_contract_errors():
    ext = build("int4gemv")
    N, K = 128, 1024
    W, s, _ = make_w4(N, K, seed=1, scale=0.02)
    X, g = _rows(2, K, seed=2)
    X, g = X.cuda(), g.cuda()
    with pytest.raises(RuntimeError, match="eps"):
        ext.forward_rmsnorm("int4gemv_rmsnorm", W, s, X, g, -1.0)
    with pytest.raises(RuntimeError, match="eps"):
        ext.forward_rmsnorm("int4gemv_rmsnorm", W, s, X, g, float("nan"))
    with pytest.raises(RuntimeError, match="unknown int4gemv_rmsnorm variant"):
        ext.forward_rmsnorm("int4gemv_mma", W, s, X, g)
    with pytest.raises(RuntimeError, match="norm_weight"):
        ext.forward_rmsnorm("int4gemv_rmsnorm", W, s, X, g[:-8])
    # a norm weight that is not 16-byte aligned: refused by the launch, no kernel runs
    gbuf = torch.empty(K + 8, dtype=torch.float16, device="cuda")
    g_odd = gbuf[1:K + 1]
    g_odd.copy_(g)
    with pytest.raises(RuntimeError, match="cudaErrorMisalignedAddress"):
        ext.forward_rmsnorm("int4gemv_rmsnorm", W, s, X, g_odd)
    assert nat.device_status(clear=True) == 0
