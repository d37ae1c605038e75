"""ctypes binding of libcudalab_gemv.so (C ABI: include/cudalab_gemv.h).

The library is the only compute path of this package.  Loading fails loudly
(RuntimeError) when it is missing; there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .build import LIB_PATH

CL_OK = 0
CL_ERR_UNKNOWN_VARIANT = 1
CL_ERR_INVALID_ARGUMENT = 2
CL_ERR_CUDA = 3
CL_ERR_BUFFER_TOO_SMALL = 4
CL_ERR_DEVICE_TIMEOUT = 5

CL_LAUNCH_PDL = 1
CL_LAUNCH_INPUTS_READY = 2
CL_LAUNCH_OUTPUTS_FREE = 4

CL_DTYPE_F16 = 0
CL_DTYPE_F32 = 1

CL_VARIANTS_NORMAL = 0
CL_VARIANTS_ALL = 1
CL_VARIANTS_QUARANTINED = 2

_lock = threading.Lock()
_lib = None

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_cs = ctypes.c_char_p
_int = ctypes.c_int
_size = ctypes.c_size_t
_dp = ctypes.POINTER(ctypes.c_double)

# name -> (restype, argtypes); every symbol declared in the public header.
PROTOTYPES = {
    "cl_version": (_cs, []),
    "cl_last_error": (_cs, []),
    "cl_device_status": (_int, [_int, ctypes.POINTER(_int)]),
    "cl_set_wait_budget": (_int, [_i64, ctypes.POINTER(_i64)]),
    "cl_int4gemv": (_int, [_cs, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "cl_int4gemv_ex": (_int, [_cs, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _u32]),
    "cl_int4gemv_native_timing": (_int, [_cs, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                         _vp, _u32, _dp]),
    "cl_int4gemv_list_variants": (_int, [_int, ctypes.c_char_p, _size, ctypes.POINTER(_size)]),
    "cl_qgemv": (_int, [_cs, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "cl_qgemv_ex": (_int, [_cs, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _u32]),
    "cl_qgemv_native_timing": (_int, [_cs, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                      _vp, _u32, _dp]),
    "cl_qgemv_list_variants": (_int, [_int, ctypes.c_char_p, _size, ctypes.POINTER(_size)]),
    "cl_peer_alloc": (_int, [_size, ctypes.POINTER(_vp), _vp]),
    "cl_peer_open": (_int, [_vp, ctypes.POINTER(_vp)]),
    "cl_peer_close": (_int, [_vp]),
    "cl_peer_free": (_int, [_vp]),
    "cl_int4gemv_sharded": (_int, [_cs, _vp, _vp, _vp, _i64, _vp, _vp, _int, _int, _i64, _i64,
                                   _i64, _i64, _vp, _u32]),
    "cl_qgemv_sharded": (_int, [_cs, _vp, _vp, _vp, _i64, _vp, _vp, _int, _int, _i64, _i64,
                                _i64, _i64, _vp, _u32]),
    "cl_int4gemv_batched": (_int, [_cs, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _u32]),
    "cl_int4gemv_quantize": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "cl_qgemv_quantize": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "cl_qgemv_batched": (_int, [_cs, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _u32]),
    "cl_int4gemv_fused_noalloc": (_int, [_cs, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _vp, _u32]),
    "cl_gemv": (_int, [_cs, _vp, _vp, _vp, _i64, _i64, _int, _vp]),
    "cl_gemv_ex": (_int, [_cs, _vp, _vp, _vp, _i64, _i64, _int, _vp, _u32]),
    "cl_gemv_native_timing": (_int, [_cs, _vp, _vp, _vp, _i64, _i64, _int, _i64, _i64, _i64, _vp,
                                     _u32, _dp]),
    "cl_gemv_list_variants": (_int, [_int, ctypes.c_char_p, _size, ctypes.POINTER(_size)]),
    "cl_rmsnorm_f16": (_int, [_vp, _vp, ctypes.c_float, _vp, _i64, _i64, _vp, _u32]),
    "cl_int4gemv_rmsnorm": (_int, [_cs, _vp, _vp, _vp, _vp, ctypes.c_float, _vp, _i64, _i64,
                                   _i64, _vp, _u32]),
}

CL_MAX_PEERS = 8
CL_IPC_HANDLE_BYTES = 64
CL_PEER_FLAG_BYTES = 64


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with typed prototypes."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build it with cudalab_b200.build.build_library() "
                "(the GEMV has no fallback path)")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def last_error(lib=None) -> str:
    lib = lib or load()
    return (lib.cl_last_error() or b"").decode("utf-8", "replace")


def list_variants(kind: str, which: int) -> list[str]:
    lib = load()
    fn = {"int4gemv": lib.cl_int4gemv_list_variants, "qgemv": lib.cl_qgemv_list_variants,
          "gemv": lib.cl_gemv_list_variants}[kind]
    needed = _size(0)
    fn(which, None, 0, ctypes.byref(needed))
    buf = ctypes.create_string_buffer(max(1, needed.value))
    rc = fn(which, buf, needed.value, ctypes.byref(needed))
    if rc != CL_OK:
        raise RuntimeError(f"list_variants failed ({rc}): {last_error(lib)}")
    text = buf.value.decode()
    return [v for v in text.split("\n") if v]


def set_wait_budget(cycles: int) -> int:
    """Bound (SM cycles) of the device-side waits of later launches; <= 0
    restores the default.  Returns the previous bound."""
    lib = load()
    prev = _i64(0)
    lib.cl_set_wait_budget(int(cycles), ctypes.byref(prev))
    return prev.value


def device_status(clear: bool = False) -> int:
    lib = load()
    out = _int(0)
    rc = lib.cl_device_status(1 if clear else 0, ctypes.byref(out))
    if rc != CL_OK:
        raise RuntimeError(f"cl_device_status failed ({rc}): {last_error(lib)}")
    return out.value
