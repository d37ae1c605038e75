"""cl_int4gemv_fused_noalloc, the entry point for callers that may not
allocate device memory (their framework owns all device allocations, or a
fixed memory budget forbids more).  It runs the fused single-GPU
step with its flag block in a fixed array inside the library; its output must
match the regular entry point, cl_int4gemv_ex, on consecutive calls (the
array keeps the previous call's contents, so a second call checks that each
call starts clean).  This file is collected last on purpose."""
import ctypes

import pytest
import torch

from cudalab_b200 import _native as nat
from cudalab_b200.build import build_library
from cudalab_b200.operators.int4gemv import make_w4, make_x4

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    build_library()
    return nat.load()


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _regular(lib, Wp, s, x, variant="int4gemv_mma"):
    N, K = Wp.shape[0], 2 * Wp.shape[1]
    y = torch.full((N,), float("nan"), dtype=torch.float16, device="cuda")
    rc = lib.cl_int4gemv_ex(variant.encode(), Wp.data_ptr(), s.data_ptr(), x.data_ptr(),
                            y.data_ptr(), N, K, _stream(), 0)
    assert rc == nat.CL_OK, nat.last_error(lib)
    return y


def _noalloc(lib, Wp, s, X, variant="int4gemv_mma", flags=0):
    N, K = Wp.shape[0], 2 * Wp.shape[1]
    M = X.shape[0] if X.dim() == 2 else 1
    y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    rc = lib.cl_int4gemv_fused_noalloc(variant.encode(), Wp.data_ptr(), s.data_ptr(),
                                       X.data_ptr(), M, y.data_ptr(), N, K, _stream(), flags)
    assert rc == nat.CL_OK, nat.last_error(lib)
    return y


def test_two_calls_match_regular_entry_point(lib):
    Wp, s, _ = make_w4(3000, 4096, seed=41, device="cuda")
    x1 = make_x4(4096, seed=42, device="cuda")
    x2 = make_x4(4096, seed=43, device="cuda")
    y1 = _noalloc(lib, Wp, s, x1)
    y2 = _noalloc(lib, Wp, s, x2, flags=nat.CL_LAUNCH_PDL | nat.CL_LAUNCH_INPUTS_READY)
    torch.cuda.synchronize()
    r1, r2 = _regular(lib, Wp, s, x1), _regular(lib, Wp, s, x2)
    torch.cuda.synchronize()
    assert torch.equal(y1[0], r1) and torch.equal(y2[0], r2)
    assert not torch.equal(y1, y2)
    assert nat.device_status(clear=True) == 0


def test_batched_rows_match(lib):
    # several activation rows: the regular batched entry point with the same
    # fixed geometry runs the same kernel apart from the stores
    Wp, s, _ = make_w4(1000, 1024, seed=44, device="cuda")
    X = torch.randn(5, 1024, generator=torch.Generator().manual_seed(45)).half().cuda()
    R = torch.full((5, 1000), float("nan"), dtype=torch.float16, device="cuda")
    rc = lib.cl_int4gemv_batched(b"int4gemv_mma_w8", Wp.data_ptr(), s.data_ptr(), X.data_ptr(),
                                 R.data_ptr(), 5, 1000, 1024, _stream(), 0)
    assert rc == nat.CL_OK, nat.last_error(lib)
    for _ in range(2):
        Y = _noalloc(lib, Wp, s, X, variant="int4gemv_mma_w8")
        torch.cuda.synchronize()
        assert torch.equal(Y, R)


def test_rejects_more_than_16_rows(lib):
    Wp, s, _ = make_w4(64, 256, seed=46, device="cuda")
    X = torch.zeros(17, 256, dtype=torch.float16, device="cuda")
    y = torch.zeros(17, 64, dtype=torch.float16, device="cuda")
    rc = lib.cl_int4gemv_fused_noalloc(b"int4gemv_mma", Wp.data_ptr(), s.data_ptr(),
                                       X.data_ptr(), 17, y.data_ptr(), 64, 256, _stream(), 0)
    assert rc == nat.CL_ERR_INVALID_ARGUMENT and "M must be in [1, 16]" in nat.last_error(lib)
