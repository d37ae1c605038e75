"""TEST INFRASTRUCTURE ONLY -- never imported by the cudalab_b200 package.

CPU restatements of the reference's weight-only quantized GEMV algorithm
(trump253/CUDALab, cudalab/int4gemv_quantize.py, cudalab/qgemv_quantize.py,
cudalab/int4gemv_correctness.py, cudalab/qgemv_correctness.py), used as the
independent checker of the CUDA path by tests/, __graft_entry__.smoke() and
the cpu_baseline / reference arm of bench.py.  Pinned against golden vectors
produced by the reference itself (tests/golden/make_golden.py).
"""
