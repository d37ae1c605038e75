"""Host-side validation of the extension objects, on CPU tensors: every check
that precedes the is_cuda check in the reference order fires with the pinned
message substring, and CPU tensors themselves are rejected as non-CUDA (the
negative suite's W_packed_cpu / W_q_cpu cases)."""
import pytest
import torch

from cudalab_b200.build import build

u8 = torch.uint8


@pytest.fixture(scope="module")
def e4():
    return build("int4gemv")


@pytest.fixture(scope="module")
def e8():
    return build("qgemv")


def _rej(fn, sub):
    with pytest.raises(RuntimeError) as ei:
        fn()
    first = str(ei.value).splitlines()[0]
    assert sub in first, first


def test_int4_order_and_messages(e4):
    N, K = 8, 256
    Wp = torch.zeros(N, K // 2, dtype=u8)
    s = torch.zeros(N, K // 128, dtype=torch.float16)
    x = torch.zeros(K, dtype=torch.float16)
    f = lambda a, b, c: e4.forward("int4gemv_baseline", a, b, c)  # noqa: E731
    _rej(lambda: e4.forward("nope", Wp, s, x), "未知 int4gemv 变体")
    _rej(lambda: f(Wp.view(-1), s, x), "必须是 2 维")
    _rej(lambda: f(torch.zeros(0, K // 2, dtype=u8), s, x), "N 必须 > 0")
    _rej(lambda: f(torch.zeros(N, 0, dtype=u8), s, x), "K/2 必须 > 0")
    _rej(lambda: f(Wp.to(torch.int8), s, x), "必须是 uint8")
    # K % 128 is checked before contiguity and device
    _rej(lambda: f(torch.zeros(N, 32, dtype=u8), s, x), "必须可被 128 整除")
    _rej(lambda: f(torch.zeros(K, N // 2, dtype=u8).t(), s, x), "连续内存")
    _rej(lambda: f(Wp, s, x), "CUDA 张量")


def test_int8_order_and_messages(e8):
    N, K = 8, 64
    Wq = torch.zeros(N, K, dtype=torch.int8)
    s = torch.zeros(N, dtype=torch.float32)
    x = torch.zeros(K, dtype=torch.float16)
    f = lambda a, b, c: e8.forward("qgemv_baseline", a, b, c)  # noqa: E731
    _rej(lambda: e8.forward("nope", Wq, s, x), "未知 qgemv 变体")
    _rej(lambda: f(Wq.view(2, 4, K), s, x), "必须是 2 维")
    _rej(lambda: f(torch.zeros(0, K, dtype=torch.int8), s, x), "N 必须 > 0")
    _rej(lambda: f(torch.zeros(N, 0, dtype=torch.int8), s, x), "K 必须 > 0")
    _rej(lambda: f(Wq.to(torch.int32), s, x), "必须是 int8")
    _rej(lambda: f(torch.zeros(K, N, dtype=torch.int8).t(), s, x), "连续内存")
    _rej(lambda: f(Wq, s, x), "CUDA 张量")


def test_variant_lists(e4, e8):
    assert e4.variants() == sorted(e4.variants())
    assert set(e4.variants()) <= set(e4.all_variants())
    for e in (e4, e8):
        assert sorted(e.variants() + e.quarantined_variants()) == e.all_variants()


# Every variant name the reference registers (kernels/int4gemv/*.cu and
# kernels/qgemv/*.cu registrars) dispatches here, so callers that name them
# (e.g. its native-timing script) run unmodified; the -m gpu suites run the
# 50-case, negative and golden checks over every listed variant.
REFERENCE_INT4 = ["int4gemv_baseline", "int4gemv_vec16_row", "int4gemv_rowtile4",
                  "int4gemv_rowtile8", "int4gemv_rowtile4_hx"]
REFERENCE_INT8 = ["qgemv_baseline", "qgemv_vec16_row", "qgemv_vec16_scale", "qgemv_warp_vec16",
                  "qgemv_warp_vec16_ilp4"]


def test_reference_variant_names_dispatch(e4, e8):
    assert set(REFERENCE_INT4) <= set(e4.variants())
    assert set(REFERENCE_INT8) <= set(e8.variants())
    assert not e4.quarantined_variants() and not e8.quarantined_variants()


def test_native_timing_result_shape():
    from cudalab_b200.ext import timing_result
    d = timing_result("int4gemv_mma", 5, 3, 8, [3.0, 1.0, 2.0])
    assert d["window_median_us"] == [3.0, 1.0, 2.0]
    assert (d["min_us"], d["median_us"], d["max_us"], d["mean_us"]) == (1.0, 2.0, 3.0, 2.0)
    assert set(d) == {"variant", "warmup", "n_windows", "launches_per_window", "window_median_us",
                      "median_us", "min_us", "max_us", "mean_us", "note"}
