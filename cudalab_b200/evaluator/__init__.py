"""Operator-agnostic evaluation helpers: fixed-tolerance correctness metrics,
the negative-case runner, benchmark pools / CUDA-graph timing and the ncu
profiler wrapper."""
