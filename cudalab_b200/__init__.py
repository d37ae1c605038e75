"""cudalab_b200: B200-native (sm_100a) weight-only quantized GEMV.

W4A16 `int4gemv` and INT8 `qgemv` behind the reference's operator API
(`build(op)` -> ext with forward / forward_into / native_timing / variants),
computed by hand-written CUDA kernels in libcudalab_gemv.so (C ABI:
include/cudalab_gemv.h).
"""
__version__ = "0.1.0"
