"""Paired A/B timing of two variants of one operator, with a fixed decision.

Role of the reference's paired harness (cudalab/evaluator/bench.py:329-549
`bench_pair`, cudalab/evaluator/stats.py:65-243, cudalab/evaluator/
decision.py): decide whether a candidate variant is faster than a parent on
one shape, with the statistical unit being the *round*, not the sample.
Back-to-back samples of one variant share clock, thermal and cache state and
are not independent; a round measures parent and candidate next to each
other on the same inputs, and rounds are what the statistics resample.

Per round (order alternates: parent first in even rounds, candidate first in
odd ones) each variant gets one block: a warm-up burn of at least
`warmup_launches` launches and `warmup_ms` of wall time, then `samples`
timed samples.  On a B200 a GEMV lasts 1-3 us, less than a host launch, so a
sample here is one replay of a CUDA graph of `launches_per_sample` launches
cycling the L2-cold pool, bracketed by CUDA events on the launching stream;
the sample's value is its time per launch.

Guards, symmetric for fast and slow outliers and identical for both variants:
  * sample guard: a sample more than `SAMPLE_GUARD` times away (either way)
    from the median of the block's last `SAMPLE_WINDOW` accepted samples is
    rejected; the block's filtered median uses the accepted samples, its raw
    median all of them;
  * block guard: after `BLOCK_WARMUP` blocks of a variant, a block whose
    filtered median is more than `BLOCK_GUARD` times away from the median of
    that variant's earlier blocks is flagged;
  * a round is valid when both blocks keep at least `MIN_ACCEPTED` samples and
    neither is flagged; an invalid round is measured again, at most
    `RETRIES` times.
Speed-up of a round = parent / candidate time (> 1: candidate faster).  Over
the valid rounds: median, mean, range, share of rounds faster, and a 95 %
percentile bootstrap interval of the median (fixed seed, so a record is
reproducible).  The same statistics on the raw medians give the raw
speed-up; when raw and filtered disagree in direction, or by more than
`SENSITIVITY` in log space, the record is marked filter-sensitive and the
decision becomes UNSTABLE whatever it was.

Decision (first rule that applies): correctness failed -> REJECT; fewer than
`MIN_VALID_ROUNDS` valid rounds -> UNSTABLE; median >= 1.05, >= 70 % of
rounds faster and CI low > 1 -> KEEP; median <= 0.95, <= 30 % faster and CI
high < 1 -> REJECT; otherwise NEUTRAL.  Separately, the statistical relation
is FASTER / SLOWER when the CI excludes 1, else UNRESOLVED.

    python -m cudalab_b200.evaluator.paired --op int4gemv --parent int4gemv_mma \
        --candidate int4gemv_mma_w4 --N 4096 --K 4096 --flags 7 --out pair.json
"""
from __future__ import annotations

import argparse
import json
import math
import statistics
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Optional, Sequence

import numpy as np

# ---- fixed parameters of the method -------------------------------------
SAMPLE_GUARD = 1.5
SAMPLE_WINDOW = 50
BLOCK_GUARD = 1.15
BLOCK_WARMUP = 3
MIN_ACCEPTED = 50
RETRIES = 3
ROUNDS = 9
MIN_VALID_ROUNDS = 5
SAMPLES = 100
LAUNCHES_PER_SAMPLE = 32
WARMUP_LAUNCHES = 150
WARMUP_MS = 300.0
BOOT_N = 10000
BOOT_SEED = 20260919
ALPHA = 0.05
SENSITIVITY = math.log(1.10)
KEEP_MEDIAN, REJECT_MEDIAN = 1.05, 0.95
KEEP_FASTER, REJECT_FASTER = 0.70, 0.30
KEEP, REJECT, NEUTRAL, UNSTABLE = "KEEP", "REJECT", "NEUTRAL", "UNSTABLE"
FASTER, SLOWER, UNRESOLVED = "FASTER", "SLOWER", "UNRESOLVED"


# ---- statistics (no GPU) ------------------------------------------------
@dataclass
class Block:
    """One variant's block of samples (us per launch) after the sample guard."""
    raw: list
    accepted: list = field(default_factory=list)
    rejected_fast: int = 0
    rejected_slow: int = 0

    @property
    def median(self) -> Optional[float]:
        return statistics.median(self.accepted) if self.accepted else None

    @property
    def raw_median(self) -> Optional[float]:
        return statistics.median(self.raw) if self.raw else None

    def as_dict(self) -> dict:
        return {"median_us": self.median, "raw_median_us": self.raw_median,
                "n_raw": len(self.raw), "n_accepted": len(self.accepted),
                "n_rejected_fast": self.rejected_fast, "n_rejected_slow": self.rejected_slow,
                "raw_samples_us": [round(v, 4) for v in self.raw]}


def outlier_side(value: float, ref: float, factor: float) -> Optional[str]:
    """'slow' / 'fast' when value is more than `factor` times away from ref
    (strictly), None otherwise."""
    if value > ref * factor:
        return "slow"
    if value * factor < ref:
        return "fast"
    return None


def guard_block(samples: Sequence[float], factor: float = SAMPLE_GUARD,
                window: int = SAMPLE_WINDOW) -> Block:
    """Apply the sample guard in arrival order; the first sample is always
    accepted (there is nothing to compare it with)."""
    b = Block(raw=list(samples))
    for v in samples:
        side = outlier_side(v, statistics.median(b.accepted[-window:]), factor) \
            if b.accepted else None
        if side is None:
            b.accepted.append(v)
        elif side == "fast":
            b.rejected_fast += 1
        else:
            b.rejected_slow += 1
    return b


def block_consistency(history: list, med: Optional[float], factor: float = BLOCK_GUARD,
                      warmup: int = BLOCK_WARMUP) -> dict:
    """Compare a block's median with the median of the variant's earlier
    blocks (`history`, appended to here); no verdict during the first
    `warmup` blocks or without a median."""
    out = {"reference_us": None, "ratio": None, "flagged": False, "direction": None}
    if med is None:
        return out
    if len(history) >= warmup:
        ref = statistics.median(history)
        out["reference_us"] = round(ref, 4)
        out["ratio"] = round(med / ref, 5) if ref > 0 else None
        side = outlier_side(med, ref, factor)
        out["flagged"] = side is not None
        out["direction"] = side
    history.append(med)
    return out


def describe(speedups: Sequence[float]) -> dict:
    if not speedups:
        return {"n": 0, "median": None, "mean": None, "min": None, "max": None,
                "faster_count": 0, "faster_fraction": None}
    a = np.asarray(speedups, dtype=np.float64)
    faster = int((a > 1.0).sum())
    return {"n": int(a.size), "median": float(np.median(a)), "mean": float(a.mean()),
            "min": float(a.min()), "max": float(a.max()), "faster_count": faster,
            "faster_fraction": faster / a.size}


def bootstrap_median_ci(values: Sequence[float], n_boot: int = BOOT_N, alpha: float = ALPHA,
                        seed: int = BOOT_SEED) -> Optional[list]:
    """Percentile bootstrap interval of the median (None below 3 values):
    n_boot resamples with replacement drawn from one seeded generator."""
    a = np.asarray(values, dtype=np.float64)
    if a.size < 3:
        return None
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, a.size, size=(n_boot, a.size))
    meds = np.sort(np.median(a[idx], axis=1))
    lo = meds[int(math.floor(alpha / 2 * n_boot))]
    hi = meds[int(math.ceil((1 - alpha / 2) * n_boot)) - 1]
    return [float(lo), float(hi)]


def filter_sensitivity(raw: Optional[float], filtered: Optional[float],
                       limit: float = SENSITIVITY) -> tuple:
    """(sensitive, reason): the guards changed the conclusion when raw and
    filtered speed-ups sit on opposite sides of 1 or differ by more than
    `limit` in log space."""
    if not raw or not filtered or raw <= 0 or filtered <= 0:
        return False, "not evaluated (missing speed-up)"
    if (raw - 1.0) * (filtered - 1.0) < 0:
        return True, f"direction differs: raw {raw:.4f}, filtered {filtered:.4f}"
    d = abs(math.log(filtered / raw))
    if d > limit:
        return True, f"|log(filtered / raw)| = {d:.4f} > {limit:.4f}"
    return False, f"|log(filtered / raw)| = {d:.4f} <= {limit:.4f}"


def decide(correctness_pass: bool, valid_rounds: int, speedups: Sequence[float],
           ci: Optional[list], sensitive: bool = False) -> dict:
    s = describe(speedups)
    if not correctness_pass:
        d, rule = REJECT, "correctness failed"
    elif valid_rounds < MIN_VALID_ROUNDS:
        d, rule = UNSTABLE, f"{valid_rounds} valid rounds < {MIN_VALID_ROUNDS}"
    elif s["median"] is None:
        d, rule = UNSTABLE, "no valid speed-up"
    elif (s["median"] >= KEEP_MEDIAN and s["faster_fraction"] >= KEEP_FASTER
          and ci is not None and ci[0] > 1.0):
        d, rule = KEEP, (f"median {s['median']:.4f} >= {KEEP_MEDIAN}, "
                         f"{s['faster_count']}/{s['n']} faster, CI low {ci[0]:.4f} > 1")
    elif (s["median"] <= REJECT_MEDIAN and s["faster_fraction"] <= REJECT_FASTER
          and ci is not None and ci[1] < 1.0):
        d, rule = REJECT, (f"median {s['median']:.4f} <= {REJECT_MEDIAN}, "
                           f"{s['faster_count']}/{s['n']} faster, CI high {ci[1]:.4f} < 1")
    else:
        d, rule = NEUTRAL, f"median {s['median']:.4f} between the thresholds or CI inconclusive"
    out = {"decision": d, "rule": rule, "original_decision": d}
    if sensitive and d != UNSTABLE:
        out["decision"] = UNSTABLE
        out["rule"] = "filter-sensitive record: " + rule
    return out


def relation(ci: Optional[list]) -> str:
    if ci is None:
        return UNRESOLVED
    if ci[0] > 1.0:
        return FASTER
    if ci[1] < 1.0:
        return SLOWER
    return UNRESOLVED


# ---- the round loop (measurement injected) ------------------------------
def run_rounds(measure: Callable[[str], list], parent: str, candidate: str,
               rounds: int = ROUNDS, retries: int = RETRIES,
               min_accepted: int = MIN_ACCEPTED) -> dict:
    """Alternate the two variants over `rounds` rounds; `measure(variant)`
    returns one block of samples (us per launch).  Returns the statistics
    record (without the correctness verdict)."""
    history = {parent: [], candidate: []}
    out_rounds = []
    for slot in range(rounds):
        order = (parent, candidate) if slot % 2 == 0 else (candidate, parent)
        rec = None
        for attempt in range(retries + 1):
            blocks = {v: guard_block(measure(v)) for v in order}
            cons = {v: block_consistency(history[v], blocks[v].median) for v in order}
            enough = all(len(blocks[v].accepted) >= min_accepted for v in order)
            steady = not any(cons[v]["flagged"] for v in order)
            bp, bc = blocks[parent], blocks[candidate]
            rec = {"round": slot + 1, "order": list(order), "retries": attempt,
                   "parent_us": bp.median, "candidate_us": bc.median,
                   "parent_raw_us": bp.raw_median, "candidate_raw_us": bc.raw_median,
                   "valid": enough and steady,
                   "invalid_reason": None if enough and steady
                   else ("too few accepted samples" if not enough else "block guard"),
                   "blocks": {"parent": bp.as_dict(), "candidate": bc.as_dict()},
                   "block_guard": {"parent": cons[parent], "candidate": cons[candidate]}}
            if rec["valid"]:
                break
        out_rounds.append(rec)
    valid = [r for r in out_rounds if r["valid"]]
    filt = [r["parent_us"] / r["candidate_us"] for r in valid]
    raw = [r["parent_raw_us"] / r["candidate_raw_us"] for r in valid]
    s_f, s_r = describe(filt), describe(raw)
    ci_f, ci_r = bootstrap_median_ci(filt), bootstrap_median_ci(raw)
    sensitive, why = filter_sensitivity(s_r["median"], s_f["median"])
    return {"parent": parent, "candidate": candidate, "n_rounds": len(out_rounds),
            "valid_rounds": len(valid), "rounds": out_rounds,
            "speedups": filt, "summary": s_f, "bootstrap_ci_95": ci_f,
            "raw": {"speedups": raw, "summary": s_r, "bootstrap_ci_95": ci_r},
            "filter_sensitive": sensitive, "filter_sensitive_reason": why,
            "parent_median_us": statistics.median([r["parent_us"] for r in valid])
            if valid else None,
            "candidate_median_us": statistics.median([r["candidate_us"] for r in valid])
            if valid else None,
            "method": {"sample_guard": SAMPLE_GUARD, "sample_window": SAMPLE_WINDOW,
                       "block_guard": BLOCK_GUARD, "block_warmup": BLOCK_WARMUP,
                       "min_accepted": min_accepted, "retries": retries,
                       "bootstrap": {"n": BOOT_N, "seed": BOOT_SEED, "alpha": ALPHA}}}


# ---- B200 measurement ---------------------------------------------------
class GraphBlocks:
    """Blocks of graph-replay samples for the variants of one pool: per
    variant one CUDA graph of `launches` launches cycling the pool (captured
    on first use), timed replay by replay with events on its stream."""

    def __init__(self, pool, ext, flags: int, launches: int = LAUNCHES_PER_SAMPLE,
                 samples: int = SAMPLES, warmup_launches: int = WARMUP_LAUNCHES,
                 warmup_ms: float = WARMUP_MS):
        import torch
        self.torch = torch
        self.pool, self.ext, self.flags = pool, ext, flags
        self.launches, self.samples = launches, samples
        self.warmup_launches, self.warmup_ms = warmup_launches, warmup_ms
        self.stream = torch.cuda.Stream()
        self.graphs = {}
        self.start = [torch.cuda.Event(enable_timing=True) for _ in range(samples)]
        self.end = [torch.cuda.Event(enable_timing=True) for _ in range(samples)]

    def _graph(self, variant: str):
        g = self.graphs.get(variant)
        if g is None:
            torch, s = self.torch, self.stream
            with torch.cuda.stream(s):
                for i in range(self.launches):  # first calls: attributes, lazy loading
                    self.pool.launch(self.ext, variant, i, flags=self.flags)
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for i in range(self.launches):
                    self.pool.launch(self.ext, variant, i, flags=self.flags)
            self.graphs[variant] = g
        return g

    def __call__(self, variant: str) -> list:
        torch, s = self.torch, self.stream
        g = self._graph(variant)
        t0, n = time.perf_counter(), 0
        with torch.cuda.stream(s):
            while n < self.warmup_launches or (time.perf_counter() - t0) * 1e3 < self.warmup_ms:
                g.replay()
                n += self.launches
                if n % (64 * self.launches) == 0:
                    s.synchronize()  # keep the burn in wall time, not in the queue
            for a, b in zip(self.start, self.end):
                a.record(s)
                g.replay()
                b.record(s)
        s.synchronize()
        return [a.elapsed_time(b) * 1e3 / self.launches for a, b in zip(self.start, self.end)]


def paired(op_name: str, parent: str, candidate: str, N: int, K: int, flags: int = 0,
           rounds: int = ROUNDS, samples: int = SAMPLES, launches: int = LAUNCHES_PER_SAMPLE,
           pool_size: int = 64, check: bool = True) -> dict:
    """Paired record of `candidate` against `parent` on an L2-cold pool of
    N x K weight sets (one activation row)."""
    import torch
    from cudalab_b200.build import build
    from cudalab_b200.operators import get
    op, ext = get(op_name), build(op_name)
    correct = True
    if check:
        from cudalab_b200 import int4gemv_correctness as c4, qgemv_correctness as c8
        mod = c4 if op_name == "int4gemv" else c8
        correct = all(r.passed for r in mod.run_suite(candidate, ext))
    pool = op.make_bench_pool(N, K, mode="l2cold", pool_size=pool_size, weight_dist=0.02)
    blocks = GraphBlocks(pool, ext, flags, launches=launches, samples=samples)
    rec = run_rounds(blocks, parent, candidate, rounds=rounds,
                     min_accepted=min(MIN_ACCEPTED, samples // 2))
    dec = decide(correct, rec["valid_rounds"], rec["speedups"], rec["bootstrap_ci_95"],
                 rec["filter_sensitive"])
    rec.update({"operator": op_name, "shape": [N, K], "flags": flags,
                "pool": {"size": pool_size, "mode": "l2cold"},
                "samples_per_block": samples, "launches_per_sample": launches,
                "correctness_pass": correct, "decision": dec,
                "statistical_relation": relation(rec["bootstrap_ci_95"]),
                "device": torch.cuda.get_device_name()})
    del blocks, pool
    return rec


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--op", default="int4gemv", choices=["int4gemv", "qgemv"])
    ap.add_argument("--parent", required=True)
    ap.add_argument("--candidate", required=True)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--flags", type=int, default=0)
    ap.add_argument("--rounds", type=int, default=ROUNDS)
    ap.add_argument("--samples", type=int, default=SAMPLES)
    ap.add_argument("--launches", type=int, default=LAUNCHES_PER_SAMPLE)
    ap.add_argument("--no-check", action="store_true")
    ap.add_argument("--out", type=Path)
    a = ap.parse_args(argv)
    rec = paired(a.op, a.parent, a.candidate, a.N, a.K, a.flags, a.rounds, a.samples,
                 a.launches, check=not a.no_check)
    text = json.dumps(rec, indent=1)
    if a.out:
        a.out.write_text(text)
    print(json.dumps({k: rec[k] for k in ("parent", "candidate", "valid_rounds",
                                          "parent_median_us", "candidate_median_us",
                                          "bootstrap_ci_95", "statistical_relation",
                                          "decision")}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
