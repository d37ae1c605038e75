"""The C-ABI library without a GPU: it loads, exports every symbol the public
header declares, lists variants, and rejects bad arguments with the right
status codes before touching any device."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from cudalab_b200 import _native as nat
from cudalab_b200.build import build_library

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    build_library()
    return nat.load()


def _declared_symbols():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(cl_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_symbols_exported(lib):
    syms = _declared_symbols()
    assert "cl_int4gemv" in syms and "cl_qgemv" in syms
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/ but not exported"
        assert s in nat.PROTOTYPES, f"{s} has no ctypes prototype"


def test_version_and_variants(lib):
    assert b"sm_100a" in lib.cl_version()
    v4 = nat.list_variants("int4gemv", nat.CL_VARIANTS_NORMAL)
    v8 = nat.list_variants("qgemv", nat.CL_VARIANTS_NORMAL)
    assert "int4gemv_baseline" in v4 and "int4gemv_bulk" in v4 and v4 == sorted(v4)
    assert "qgemv_baseline" in v8 and "qgemv_bulk" in v8 and v8 == sorted(v8)
    for kind, normal in (("int4gemv", v4), ("qgemv", v8)):
        allv = nat.list_variants(kind, nat.CL_VARIANTS_ALL)
        quar = nat.list_variants(kind, nat.CL_VARIANTS_QUARANTINED)
        assert allv == sorted(normal + quar) and not set(normal) & set(quar)


def test_list_variants_buffer_contract(lib):
    needed = ctypes.c_size_t(0)
    rc = lib.cl_int4gemv_list_variants(nat.CL_VARIANTS_NORMAL, None, 0, ctypes.byref(needed))
    assert rc == nat.CL_ERR_BUFFER_TOO_SMALL and needed.value > 1
    buf = ctypes.create_string_buffer(needed.value)
    assert lib.cl_int4gemv_list_variants(nat.CL_VARIANTS_NORMAL, buf, needed.value,
                                         ctypes.byref(needed)) == nat.CL_OK
    assert lib.cl_int4gemv_list_variants(7, buf, needed.value, None) == nat.CL_ERR_INVALID_ARGUMENT


def test_status_codes_without_device(lib):
    # unknown variant is reported before any argument or device work
    rc = lib.cl_int4gemv(b"no_such", None, None, None, None, 4, 128, None)
    assert rc == nat.CL_ERR_UNKNOWN_VARIANT
    assert "no_such" in nat.last_error(lib)
    # N <= 0, K % 128 != 0, null pointers: rejected on the host
    assert lib.cl_int4gemv(b"int4gemv_baseline", None, None, None, None, 0, 128, None) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert lib.cl_int4gemv(b"int4gemv_bulk", None, None, None, None, 4, 64, None) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert "128" in nat.last_error(lib)
    assert lib.cl_int4gemv(b"int4gemv_bulk", None, None, None, None, 4, 128, None) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert lib.cl_qgemv(b"qgemv_baseline", None, None, None, None, 4, 0, None) == \
        nat.CL_ERR_INVALID_ARGUMENT
    buf = (ctypes.c_double * 2)()
    assert lib.cl_qgemv_native_timing(b"qgemv_ldg", None, None, None, None, 4, 16, -1, 2, 4,
                                      None, 0, buf) == nat.CL_ERR_INVALID_ARGUMENT


def test_noalloc_entry_rejects_before_device_work(lib):
    # the allocation-free fused step validates everything before it looks up
    # its device array or touches the stream, so these run without a GPU
    fake = 1 << 20  # a 16-byte aligned, never dereferenced address
    f = lib.cl_int4gemv_fused_noalloc
    assert f(b"no_such", fake, fake, fake, 1, fake, 64, 256, None, 0) == \
        nat.CL_ERR_UNKNOWN_VARIANT
    assert f(b"int4gemv_mma", fake, fake, fake, 17, fake, 64, 256, None, 0) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert "[1, 16]" in nat.last_error(lib)
    assert f(b"int4gemv_mma", fake, fake, fake, 1, None, 64, 256, None, 0) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert f(b"int4gemv_mma", fake, fake, fake, 1, fake, 64, 200, None, 0) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert f(b"int4gemv_mma", fake + 2, fake, fake, 1, fake, 64, 256, None, 0) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert "16-byte" in nat.last_error(lib)


def test_rmsnorm_entries_reject_before_device_work(lib):
    # every host-side contract check of the RMSNorm and fused entry points
    # returns before the first CUDA call, so these run without a GPU
    fake = 1 << 20
    r = lib.cl_rmsnorm_f16
    assert r(fake, fake, 1e-5, fake, 0, 64, None, 0) == nat.CL_ERR_INVALID_ARGUMENT
    assert r(fake, fake, 1e-5, fake, 2, 60, None, 0) == nat.CL_ERR_INVALID_ARGUMENT
    assert "multiple of 8" in nat.last_error(lib)
    assert r(fake, fake, 1e-5, fake, 2, 4 << 20, None, 0) == nat.CL_ERR_INVALID_ARGUMENT
    assert r(fake, fake, -1.0, fake, 2, 64, None, 0) == nat.CL_ERR_INVALID_ARGUMENT
    assert r(fake, fake, float("inf"), fake, 2, 64, None, 0) == nat.CL_ERR_INVALID_ARGUMENT
    assert "eps" in nat.last_error(lib)
    assert r(None, fake, 1e-5, fake, 2, 64, None, 0) == nat.CL_ERR_INVALID_ARGUMENT
    f = lib.cl_int4gemv_rmsnorm
    assert f(b"int4gemv_mma", fake, fake, fake, fake, 1e-5, fake, 1, 64, 256, None, 0) == \
        nat.CL_ERR_UNKNOWN_VARIANT
    assert f(b"int4gemv_rmsnorm", fake, fake, fake, fake, 1e-5, fake, 0, 64, 256, None, 0) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert f(b"int4gemv_rmsnorm", fake, fake, fake, fake, 1e-5, fake, 1, 64, 200, None, 0) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert "128" in nat.last_error(lib)
    assert f(b"int4gemv_rmsnorm", fake, fake, fake, None, 1e-5, fake, 1, 64, 256, None, 0) == \
        nat.CL_ERR_INVALID_ARGUMENT
    assert f(b"int4gemv_rmsnorm", fake, fake, fake, fake, float("nan"), fake, 1, 64, 256, None,
             0) == nat.CL_ERR_INVALID_ARGUMENT


def test_product_has_no_oracle_dependency():
    """The package never imports the checker (oracle/)."""
    pkg = ROOT / "cudalab_b200"
    for f in pkg.rglob("*.py"):
        text = f.read_text()
        assert "import oracle" not in text and "from oracle" not in text, f


def test_library_is_sm100a_build():
    stamp = (ROOT / "cudalab_b200" / "_lib" / "libcudalab_gemv.stamp.json").read_text()
    assert "compute_100a" in stamp and "sm_100a" in stamp


def test_torch_cpu_only_here_or_gpu():
    # documents the environment split: this file never needs a device
    assert isinstance(torch.cuda.is_available(), bool)


def test_wait_budget_roundtrip(lib):
    """The device-wait bound is host state: set, read back, and restored to
    the default by a non-positive value (no device work)."""
    prev = nat.set_wait_budget(12345)
    try:
        assert nat.set_wait_budget(777) == 12345
        assert nat.set_wait_budget(0) == 777
        assert nat.set_wait_budget(0) == 4_000_000_000  # the default
    finally:
        nat.set_wait_budget(prev)
