"""The paired timing engine's statistics and round logic, on synthetic samples
(no GPU): symmetric guards with strict thresholds, the block guard's warm-up,
a reproducible bootstrap that covers the median, the filter-sensitivity rule,
the fixed decision table, and the round loop's ordering, retries and
speed-up bookkeeping with an injected measurement."""
import math

import numpy as np
import pytest

from cudalab_b200.evaluator import paired as pr


def test_outlier_side_symmetric_and_strict():
    assert pr.outlier_side(15.0, 10.0, 1.5) is None          # exactly at the bound
    assert pr.outlier_side(15.0001, 10.0, 1.5) == "slow"
    assert pr.outlier_side(10.0 / 1.5, 10.0, 1.5) is None
    assert pr.outlier_side(6.6, 10.0, 1.5) == "fast"


def test_guard_block_rejects_both_sides():
    samples = [10.0] * 20 + [30.0, 2.0] + [10.1] * 5
    b = pr.guard_block(samples)
    assert b.rejected_slow == 1 and b.rejected_fast == 1
    assert len(b.accepted) == len(samples) - 2
    assert b.median == pytest.approx(10.0) and b.raw_median == pytest.approx(10.0)
    # the first sample is always accepted
    assert pr.guard_block([100.0, 10.0]).accepted == [100.0]


def test_guard_window_follows_recent_samples():
    # a level shift that the window absorbs step by step is accepted
    samples = [10.0 * (1.1 ** i) for i in range(30)]
    assert pr.guard_block(samples, window=3).rejected_slow == 0


def test_block_consistency_warmup_and_direction():
    hist = []
    for v in (10.0, 10.2, 9.9):
        assert not pr.block_consistency(hist, v)["flagged"]
    slow = pr.block_consistency(hist, 12.0)
    assert slow["flagged"] and slow["direction"] == "slow"
    fast = pr.block_consistency(hist, 8.0)
    assert fast["flagged"] and fast["direction"] == "fast"
    ok = pr.block_consistency(hist, 10.1)
    assert not ok["flagged"] and len(hist) == 6
    assert pr.block_consistency(hist, None)["flagged"] is False and len(hist) == 6


def test_bootstrap_reproducible_and_brackets_median():
    rng = np.random.default_rng(5)
    vals = list(1.0 + 0.02 * rng.standard_normal(15))
    a = pr.bootstrap_median_ci(vals)
    b = pr.bootstrap_median_ci(vals)
    assert a == b
    assert a[0] <= float(np.median(vals)) <= a[1]
    assert pr.bootstrap_median_ci([1.0, 1.1]) is None
    assert pr.bootstrap_median_ci([2.0, 2.0, 2.0]) == [2.0, 2.0]


def test_filter_sensitivity_rules():
    assert pr.filter_sensitivity(0.98, 1.02)[0]               # direction flip
    assert pr.filter_sensitivity(1.02, 1.15)[0]               # > 10 % apart
    assert not pr.filter_sensitivity(1.02, 1.05)[0]
    assert not pr.filter_sensitivity(None, 1.05)[0]
    assert pr.SENSITIVITY == pytest.approx(math.log(1.10))


@pytest.mark.parametrize("speedups,ci,expected", [
    ([1.10] * 7, [1.08, 1.12], pr.KEEP),
    ([0.90] * 7, [0.88, 0.92], pr.REJECT),
    ([1.02] * 7, [1.01, 1.03], pr.NEUTRAL),                  # below the 5 % threshold
    ([1.10] * 4 + [0.99] * 3, [0.99, 1.10], pr.NEUTRAL),      # CI includes 1
    ([1.10] * 4, [1.08, 1.12], pr.UNSTABLE),                  # too few valid rounds
])
def test_decision_table(speedups, ci, expected):
    assert pr.decide(True, len(speedups), speedups, ci)["decision"] == expected


def test_decision_correctness_and_sensitivity():
    assert pr.decide(False, 9, [1.2] * 9, [1.1, 1.3])["decision"] == pr.REJECT
    d = pr.decide(True, 9, [1.2] * 9, [1.1, 1.3], sensitive=True)
    assert d["decision"] == pr.UNSTABLE and d["original_decision"] == pr.KEEP
    assert pr.relation([1.01, 1.2]) == pr.FASTER
    assert pr.relation([0.8, 0.99]) == pr.SLOWER
    assert pr.relation([0.99, 1.01]) == pr.UNRESOLVED and pr.relation(None) == pr.UNRESOLVED


def _fake_measure(times, n=60, noisy_round=None):
    calls = []
    rng = np.random.default_rng(0)

    def measure(variant):
        calls.append(variant)
        base = times[variant]
        if noisy_round is not None and len(calls) in noisy_round:
            base *= 1.5  # a uniformly slow block: caught by the block guard
        return list(base * (1.0 + 0.005 * rng.standard_normal(n)))
    return measure, calls


def test_round_loop_alternates_and_decides():
    measure, calls = _fake_measure({"a": 2.0, "b": 1.6})
    rec = pr.run_rounds(measure, "a", "b", rounds=7)
    assert calls[:4] == ["a", "b", "b", "a"]                   # parent first in even rounds
    assert rec["valid_rounds"] == 7
    assert rec["summary"]["median"] == pytest.approx(1.25, rel=0.01)
    d = pr.decide(True, rec["valid_rounds"], rec["speedups"], rec["bootstrap_ci_95"],
                  rec["filter_sensitive"])
    assert d["decision"] == pr.KEEP and pr.relation(rec["bootstrap_ci_95"]) == pr.FASTER


def test_round_loop_retries_a_flagged_round():
    # blocks 9 and 10 (round 5: warm-up of 3 blocks per variant is over) are slow
    measure, calls = _fake_measure({"a": 2.0, "b": 2.0}, noisy_round={9, 10})
    rec = pr.run_rounds(measure, "a", "b", rounds=6)
    r5 = rec["rounds"][4]
    assert r5["retries"] == 1 and r5["valid"]
    assert rec["valid_rounds"] == 6 and len(calls) == 14
    d = pr.decide(True, rec["valid_rounds"], rec["speedups"], rec["bootstrap_ci_95"])
    assert d["decision"] == pr.NEUTRAL


def test_round_loop_too_few_samples_is_unstable():
    measure, _ = _fake_measure({"a": 2.0, "b": 1.0}, n=10)
    rec = pr.run_rounds(measure, "a", "b", rounds=5, retries=1)
    assert rec["valid_rounds"] == 0
    assert pr.decide(True, 0, rec["speedups"], rec["bootstrap_ci_95"])["decision"] == pr.UNSTABLE
