"""Operator adapter registry (mirror of cudalab/operators/__init__.py:17-29,
restricted to the quantized GEMV operators of this package)."""
from __future__ import annotations

from .int4gemv import int4gemv as _int4gemv
from .qgemv import qgemv as _qgemv

_REGISTRY = {op.name: op for op in (_qgemv, _int4gemv)}


def get(name: str):
    try:
        return _REGISTRY[name]
    except KeyError:
        raise KeyError(f"unknown operator {name!r}; available: {sorted(_REGISTRY)}") from None


def names() -> list[str]:
    return sorted(_REGISTRY)
