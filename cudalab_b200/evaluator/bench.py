"""Benchmark pools and device-side timing.

Role of cudalab/evaluator/bench.py (BenchPool :190-233, measure_block
:259-311, time_call :772).  On a B200 one GEMV launch lasts 1-3 us, so a
Python loop of launches is host-bound; the timings here therefore come from
CUDA graphs (a whole pass over a pool captured once, replayed) or from the
library's native C++ launch loop, always with CUDA events recorded on the
launching stream.
"""
from __future__ import annotations

import statistics
from dataclasses import dataclass, field
from typing import Callable, Optional

import torch

SEED = 1234
POOL_SIZE = 16


@dataclass
class BenchPool:
    """Pre-allocated tensors of a timed region; `launch(ext, variant, i,
    flags=0)` issues launch number i (rotation is the pool's business)."""
    xs: list
    outs: list
    pool_size: int
    working_set_bytes: int
    element_size: int
    mode: str
    launch: Callable = field(repr=False)
    shared: dict = field(default_factory=dict, repr=False)
    shared_bytes: int = 0
    pool_extra: dict = field(default_factory=dict)

    def __post_init__(self):
        if self.mode not in ("hot", "streaming", "l2cold"):
            raise ValueError(f"unknown cache mode: {self.mode}")
        if self.mode == "hot" and (len(self.xs) != 1 or len(self.outs) != 1):
            raise ValueError("hot mode needs exactly one x/out buffer")


def _median(v):
    return statistics.median(v) if v else float("nan")


def graph_timing(pool: BenchPool, ext, variant: str, launches: int, replays: int,
                 warmup_replays: int = 3, flags: int = 0,
                 stream: Optional[torch.cuda.Stream] = None) -> dict:
    """Capture `launches` consecutive pool launches in one CUDA graph and time
    `replays` replays with CUDA events on the replay stream.  Returns
    per-launch microseconds for each replay plus summary statistics."""
    s = stream or torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for i in range(launches):  # eager warm-up: module load, smem attributes
            pool.launch(ext, variant, i, flags=flags)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(launches):
            pool.launch(ext, variant, i, flags=flags)
    with torch.cuda.stream(s):
        for _ in range(warmup_replays):
            g.replay()
    s.synchronize()
    per = []
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        for _ in range(replays):
            e0.record(s)
            g.replay()
            e1.record(s)
            e1.synchronize()
            per.append(e0.elapsed_time(e1) * 1e3 / launches)
    del g
    return {"per_launch_us": per, "median_us": _median(per), "min_us": min(per),
            "max_us": max(per), "launches_per_graph": launches, "replays": replays,
            "flags": flags}


def time_call(fn: Callable[[], object], warmup: int = 100, iters: int = 200,
              batch: int = 32) -> dict:
    """API-path timing of a Python callable: events around `batch` calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    per = []
    for _ in range(iters):
        e0.record()
        for _ in range(batch):
            fn()
        e1.record()
        e1.synchronize()
        per.append(e0.elapsed_time(e1) * 1e3 / batch)
    return {"median_us": _median(per), "min_us": min(per), "max_us": max(per),
            "iters": iters, "batch": batch}
