"""INT4 parity tests on the GPU (through the C ABI via the extension object).

  * the 50-case layer-A suite (10 shapes x 5 modes) per variant;
  * the 30-case negative suite per variant;
  * the reference's golden vectors (tests/golden) on every variant;
  * full-size north-star shapes (4096x4096, the 7B sweep, the 70B MLP shapes) against the numpy oracle's fixed bound;
  * determinism, PDL launches, CUDA-graph capture, native timing.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from cudalab_b200 import _native as nat
from cudalab_b200.build import build
from cudalab_b200.int4gemv_correctness import run_suite, summarize
from cudalab_b200.int4gemv_negative import run_negative_suite
from cudalab_b200.operators.int4gemv import make_w4, make_x4
from oracle import int4gemv_oracle as orc

pytestmark = pytest.mark.gpu
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "int4gemv_golden.npz")


@pytest.fixture(scope="module")
def ext():
    return build("int4gemv")


def _variants():
    return nat.list_variants("int4gemv", nat.CL_VARIANTS_NORMAL)


@pytest.mark.parametrize("variant", _variants())
def test_layer_a_suite(ext, variant):
    res = run_suite(variant, ext)
    s = summarize(res)
    bad = [(r.shape, r.mode, r.arith_max_ratio) for r in res if not r.passed]
    assert s["all_pass"] and s["n_total"] == 50, bad
    assert nat.device_status(clear=True) == 0


@pytest.mark.parametrize("variant", _variants())
def test_negative_suite(ext, variant):
    doc = run_negative_suite(ext, variant=variant)
    bad = [(c["id"], c["outcome"], c["first_line"]) for c in doc["cases"] if not c.get("pass")]
    assert doc["summary"]["all_pass"] and doc["summary"]["n_total"] == 30, bad


@pytest.mark.parametrize("variant", _variants())
def test_golden_vectors(ext, variant):
    for i in range(int(GOLD["n_cases"])):
        p = f"c{i}_"
        Wp = torch.from_numpy(GOLD[p + "W_packed"]).cuda()
        s = torch.from_numpy(GOLD[p + "scale"].view(np.float16).copy()).cuda()
        x = torch.from_numpy(GOLD[p + "x"].view(np.float16).copy()).cuda()
        y = ext.forward(variant, Wp, s, x).cpu().numpy()
        K = 2 * Wp.shape[1]
        ratio = orc.arith_ratio(y, K, GOLD[p + "exact"], GOLD[p + "S"])
        assert np.isfinite(y.astype(np.float32)).all()
        assert ratio <= 1.0, (i, ratio)


FULL = [(4096, 4096), (1024, 4096), (4096, 1024), (11008, 4096), (4096, 11008)]


@pytest.mark.parametrize("shape", FULL, ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("variant", ["int4gemv_mma", "int4gemv_mma_w4", "int4gemv_mma_w8c2",
                                     "int4gemv_mma_w4h", "int4gemv_bulk", "int4gemv_ldg"])
def test_full_size_vs_oracle(ext, variant, shape):
    N, K = shape
    Wp, s, _ = make_w4(N, K, seed=77, scale=0.02)
    x = make_x4(K, seed=78)
    y = ext.forward(variant, Wp, s, x).cpu().numpy()
    if variant == "int4gemv_mma":
        # the geometry of independent launches (flags 7) gives the same bits
        y7 = ext.forward(variant, Wp, s, x, flags=nat.CL_LAUNCH_PDL | nat.CL_LAUNCH_INPUTS_READY
                         | nat.CL_LAUNCH_OUTPUTS_FREE)
        assert np.array_equal(y7.cpu().numpy().view(np.uint16), y.view(np.uint16))
    r = orc.check(y, Wp.cpu().numpy(), s.cpu().numpy(), x.cpu().numpy())
    assert r["pass"], r


@pytest.mark.parametrize("shape", [(28672, 8192), (8192, 28672)], ids=str)
def test_sharding_shapes_row_sample(ext, shape):
    """70B-class MLP shapes: full GEMV on the device, oracle on 512 sampled rows."""
    N, K = shape
    Wp, s, _ = make_w4(N, K, seed=91, scale=0.02)
    x = make_x4(K, seed=92)
    y = ext.forward("int4gemv_mma", Wp, s, x).cpu().numpy()
    rows = np.random.default_rng(0).choice(N, 512, replace=False)
    r = orc.check(y[rows], Wp.cpu().numpy()[rows], s.cpu().numpy()[rows], x.cpu().numpy())
    assert r["pass"], r


@pytest.mark.parametrize("variant", _variants())
def test_deterministic_and_pdl_identical(ext, variant):
    Wp, s, _ = make_w4(2048, 4096, seed=5)
    x = make_x4(4096, seed=6)
    y0 = ext.forward(variant, Wp, s, x)
    y1 = ext.forward(variant, Wp, s, x)
    y2 = ext.forward(variant, Wp, s, x, flags=nat.CL_LAUNCH_PDL)
    y3 = ext.forward(variant, Wp, s, x, flags=nat.CL_LAUNCH_PDL | nat.CL_LAUNCH_INPUTS_READY)
    y4 = ext.forward(variant, Wp, s, x, flags=nat.CL_LAUNCH_PDL | nat.CL_LAUNCH_INPUTS_READY
                     | nat.CL_LAUNCH_OUTPUTS_FREE)
    assert torch.equal(y0, y1) and torch.equal(y0, y2) and torch.equal(y0, y3)
    assert torch.equal(y0, y4)


def _misaligned_copy(s: torch.Tensor) -> torch.Tensor:
    """The same scales in a contiguous tensor that starts 2 bytes past an
    8-byte boundary."""
    buf = torch.empty(s.numel() + 1, dtype=s.dtype, device=s.device)
    out = buf[1:].view(s.shape)
    out.copy_(s)
    assert out.is_contiguous() and out.data_ptr() % 8 == 2
    return out


@pytest.mark.parametrize("M", [1, 4, 16])
def test_misaligned_scales_same_bits(ext, M):
    # Scale rows that are not 8-byte aligned take the kernel's per-item address
    # path instead of the stepped vector loads; the sums are the same.
    Wp, s, _ = make_w4(1536, 4096, seed=21)
    s2 = _misaligned_copy(s)
    if M == 1:
        x = make_x4(4096, seed=22)
        for v in ("int4gemv_mma", "int4gemv_mma_w2", "int4gemv_mma_w8c2"):
            assert torch.equal(ext.forward(v, Wp, s, x), ext.forward(v, Wp, s2, x)), v
    else:
        X = torch.randn(M, 4096, generator=torch.Generator().manual_seed(23)).half().cuda()
        for v in ("int4gemv_mma", "int4gemv_mma_w8"):
            assert torch.equal(ext.forward_batched(v, Wp, s, X),
                               ext.forward_batched(v, Wp, s2, X)), v


def test_graph_capture_matches_eager(ext):
    Wps = [make_w4(1024, 2048, seed=20 + i)[:2] for i in range(4)]
    xs = [make_x4(2048, seed=40 + i) for i in range(4)]
    outs = [torch.empty(1024, dtype=torch.float16, device="cuda") for _ in range(4)]
    eager = [ext.forward("int4gemv_bulk", w, s, x) for (w, s), x in zip(Wps, xs)]
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for (w, s), x, o in zip(Wps, xs, outs):
            ext.forward_into("int4gemv_bulk", w, s, x, o, flags=nat.CL_LAUNCH_PDL)
    st.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for (w, s), x, o in zip(Wps, xs, outs):
            ext.forward_into("int4gemv_bulk", w, s, x, o, flags=nat.CL_LAUNCH_PDL)
    for o in outs:
        o.zero_()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, outs):
        assert torch.equal(a, b)
    del g


def test_native_timing(ext):
    Wp, s, _ = make_w4(4096, 4096, seed=1234)
    x = make_x4(4096, seed=1234)
    out = torch.empty(4096, dtype=torch.float16, device="cuda")
    d = ext.native_timing("int4gemv_bulk", Wp, s, x, out, 20, 3, 16)
    assert set(d) >= {"variant", "median_us", "min_us", "max_us", "mean_us", "window_median_us"}
    assert len(d["window_median_us"]) == 3 and 0 < d["min_us"] <= d["max_us"] < 1e5
    assert nat.device_status(clear=True) == 0


def _outlier_case(N, K, seed):
    """Groups whose quantised values are nearly all 0 (one outlier of about
    +-5 among weights of about 1e-3) and activations spread over six decades:
    the inputs on which a biased tensor-core operand loses the most relative
    accuracy."""
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(N, K, generator=g) * 1e-3
    idx = torch.randint(0, 128, (N, K // 128), generator=g) + torch.arange(0, K, 128)
    W.scatter_(1, idx, torch.randn(N, K // 128, generator=g).sign() * 5.0)
    mag = torch.pow(10.0, torch.randint(-3, 3, (K,), generator=g).float())
    x = (torch.randn(K, generator=g) * mag).half()
    from cudalab_b200.int4gemv_quantize import quantize_w
    Wp, s = quantize_w(W.half())
    return Wp.cuda(), s.cuda(), x.cuda()


@pytest.mark.parametrize("K", [128, 1024, 4096])
@pytest.mark.parametrize("variant", ["int4gemv_mma", "int4gemv_mma_w4", "int4gemv_mma_w8",
                                     "int4gemv_mma_w8c2", "int4gemv_mma_w16",
                                     "int4gemv_mma_w4h", "int4gemv_baseline"])
def test_outlier_groups_vs_oracle(ext, variant, K):
    Wp, s, x = _outlier_case(512, K, seed=K)
    y = ext.forward(variant, Wp, s, x).cpu().numpy()
    r = orc.check(y, Wp.cpu().numpy(), s.cpu().numpy(), x.cpu().numpy())
    assert r["pass"], r


@pytest.fixture(scope="module")
def one_rank_group():
    import torch.distributed as dist
    if dist.is_initialized():
        yield None
        return
    store = dist.HashStore()
    dist.init_process_group("gloo", store=store, rank=0, world_size=1)
    yield None
    dist.destroy_process_group()


@pytest.mark.parametrize("flags", [0, 1, 3])
@pytest.mark.parametrize("variant", ["int4gemv_mma", "int4gemv_mma_w4", "int4gemv_mma_w8",
                                     "int4gemv_mma_w8c2"])
def test_sharded_fused_single_rank(ext, one_rank_group, variant, flags):
    """The fused sharded step with one rank (the peer epilogue, the flag
    protocol and the device step counter on a single GPU) equals the plain
    GEMV bit for bit over several steps."""
    from cudalab_b200.sharded import ShardedGemv
    Wp, s, _ = make_w4(1000, 2048, seed=3)
    sg = ShardedGemv("int4gemv", Wp, s, 1000, 2048, variant=variant, mode="fused")
    try:
        for step in range(4):
            x = make_x4(2048, seed=50 + step)
            y = sg.forward(x, flags=flags).clone()
            ref = ext.forward(variant, Wp, s, x)
            torch.cuda.synchronize()
            assert torch.equal(y, ref), step
        assert nat.device_status(clear=True) == 0
    finally:
        sg.close()


@pytest.mark.parametrize("M", [1, 3, 16])
@pytest.mark.parametrize("variant", ["int4gemv_tc", "int4gemv_mma"])
def test_sharded_fused_single_rank_batches(ext, one_rank_group, variant, M):
    """Several activation rows through the fused sharded step on one rank
    (the tcgen05 kernel's peer epilogue included; "int4gemv_mma" routes 16
    rows on few tiles to it) equal the plain batched GEMV bit for bit."""
    from cudalab_b200.sharded import ShardedGemv
    Wp, s, _ = make_w4(1000, 4096, seed=5)
    sg = ShardedGemv("int4gemv", Wp, s, 1000, 4096, variant=variant, mode="fused", max_batch=16)
    try:
        for step in range(3):
            X = torch.randn(M, 4096, generator=torch.Generator().manual_seed(60 + step))
            X = X.half().cuda()
            y = sg.forward(X if M > 1 else X[0], flags=3).clone().view(M, 1000)
            ref = ext.forward_batched(variant, Wp, s, X)
            torch.cuda.synchronize()
            assert torch.equal(y, ref), step
        assert nat.device_status(clear=True) == 0
    finally:
        sg.close()


@pytest.mark.parametrize("graph", [False, True])
def test_outputs_free_chain_completes_in_order(ext, graph):
    """A chain of independent GEMVs launched with PDL | INPUTS_READY |
    OUTPUTS_FREE (only one CTA of each waits for its predecessor), a slow one
    first, then a plain consumer kernel: the consumer must see every output
    (buffers start as NaN, so a stale read is detected)."""
    flags = nat.CL_LAUNCH_PDL | nat.CL_LAUNCH_INPUTS_READY | nat.CL_LAUNCH_OUTPUTS_FREE
    shapes = [(28672, 8192)] + [(1024, 4096)] * 7
    ws = [make_w4(N, K, seed=200 + i)[:2] for i, (N, K) in enumerate(shapes)]
    xs = [make_x4(K, seed=300 + i) for i, (N, K) in enumerate(shapes)]
    ref = [ext.forward("int4gemv_mma", w, sc, x) for (w, sc), x in zip(ws, xs)]
    outs = [torch.empty(N, dtype=torch.float16, device="cuda") for N, _ in shapes]
    st = torch.cuda.Stream()

    def chain():
        for (w, sc), x, o in zip(ws, xs, outs):
            ext.forward_into("int4gemv_mma", w, sc, x, o, flags=flags)
        return torch.cat(outs)  # plain kernels reading every output

    for _ in range(3 if graph else 20):
        for o in outs:
            o.fill_(float("nan"))
        torch.cuda.synchronize()
        if graph:
            with torch.cuda.stream(st):
                chain()
            st.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                got = chain()
            for o in outs:
                o.fill_(float("nan"))
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            del g
        else:
            with torch.cuda.stream(st):
                got = chain()
            st.synchronize()
        assert torch.equal(got, torch.cat(ref))
    assert nat.device_status(clear=True) == 0
