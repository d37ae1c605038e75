"""TEST INFRASTRUCTURE ONLY: ctypes front end of oracle/cpu_gemv.c (the timed
CPU restatement of the reference's dequantise-then-mv CPU path).  Built by
`make -C oracle` into oracle/_build/libcpu_gemv.so."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libcpu_gemv.so"
_lib = None


def build() -> Path:
    subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        lib = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        for name in ("oracle_int4_gemv", "oracle_int8_gemv"):
            fn = getattr(lib, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [P, P, P, P, I64, I64, P, ctypes.c_int]
        lib.oracle_max_threads.restype = ctypes.c_int
        lib.oracle_h2f.restype = ctypes.c_float
        lib.oracle_h2f.argtypes = [ctypes.c_uint16]
        lib.oracle_f2h.restype = ctypes.c_uint16
        lib.oracle_f2h.argtypes = [ctypes.c_float]
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(load().oracle_max_threads())


class Workspace:
    """Reusable host buffers (the materialised fp32 matrix + x)."""

    def __init__(self, N: int, K: int):
        self.N, self.K = N, K
        self.work = np.empty(N * K + K, np.float32)
        self.y = np.empty(N, np.float16)


def int4_gemv(Wp: np.ndarray, scale16: np.ndarray, x16: np.ndarray, threads: int,
              ws: Workspace | None = None) -> np.ndarray:
    N, K = Wp.shape[0], 2 * Wp.shape[1]
    ws = ws or Workspace(N, K)
    rc = load().oracle_int4_gemv(Wp.ctypes.data, scale16.ctypes.data, x16.ctypes.data,
                                 ws.y.ctypes.data, N, K, ws.work.ctypes.data, threads)
    if rc:
        raise ValueError("oracle_int4_gemv rejected its arguments")
    return ws.y.copy()


def int8_gemv(Wq: np.ndarray, scale32: np.ndarray, x16: np.ndarray, threads: int,
              ws: Workspace | None = None) -> np.ndarray:
    N, K = Wq.shape
    ws = ws or Workspace(N, K)
    rc = load().oracle_int8_gemv(Wq.ctypes.data, scale32.ctypes.data, x16.ctypes.data,
                                 ws.y.ctypes.data, N, K, ws.work.ctypes.data, threads)
    if rc:
        raise ValueError("oracle_int8_gemv rejected its arguments")
    return ws.y.copy()
