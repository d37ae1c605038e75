"""Operator adapter protocol (the boundary between the evaluator and an
operator; role of cudalab/operators/base.py:40-118).

An abstract base class: an operator that leaves one of the abstract methods
out cannot be instantiated, so the registry (`operators.get`) fails at once
instead of at the first evaluator call."""
from __future__ import annotations

from abc import ABC, abstractmethod
from pathlib import Path


class Operator(ABC):
    name: str
    dtypes: tuple
    bench_shapes: list
    primary_target: tuple
    ncu_kernel_regex: str
    profiles_dir: Path

    @abstractmethod
    def build(self):
        """The built extension object (the reference's `build(<op>)`)."""

    def variants(self, ext) -> list[str]:
        return sorted(ext.variants())

    def unsafe_variants(self, ext) -> list[str]:
        fn = getattr(ext, "quarantined_variants", None)
        return sorted(fn()) if fn is not None else []

    @abstractmethod
    def make_bench_pool(self, M, H, dtype, mode, seed, pool_size):
        """A pool of independent inputs cycled call by call, and its launcher."""

    @abstractmethod
    def algorithmic_bytes(self, M: int, H: int, element_size: int = 2) -> int:
        """Bytes one call must move at minimum (weights, scales, x, y)."""

    @abstractmethod
    def experiment_prefix(self) -> str:
        """Prefix of the operator's experiment names."""

    @abstractmethod
    def run_correctness(self, ext, variant: str) -> dict:
        """The reference's correctness suite for one variant, summarised."""

    @abstractmethod
    def run_negative(self, ext, variant: str | None = None) -> dict:
        """The reference's negative suite, summarised."""
