"""Operator adapter protocol (the boundary between the evaluator and an
operator; role of cudalab/operators/base.py:40-118)."""
from __future__ import annotations

from pathlib import Path


class Operator:
    name: str
    dtypes: tuple
    bench_shapes: list
    primary_target: tuple
    ncu_kernel_regex: str
    profiles_dir: Path

    def build(self):
        raise NotImplementedError

    def variants(self, ext) -> list[str]:
        return sorted(ext.variants())

    def unsafe_variants(self, ext) -> list[str]:
        fn = getattr(ext, "quarantined_variants", None)
        return sorted(fn()) if fn is not None else []

    def make_bench_pool(self, M, H, dtype, mode, seed, pool_size):
        raise NotImplementedError

    def algorithmic_bytes(self, M: int, H: int, element_size: int = 2) -> int:
        raise NotImplementedError

    def experiment_prefix(self) -> str:
        raise NotImplementedError

    def run_correctness(self, ext, variant: str) -> dict:
        raise NotImplementedError

    def run_negative(self, ext, variant: str | None = None) -> dict:
        raise NotImplementedError
