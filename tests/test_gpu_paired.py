"""The paired timing engine on a B200, shortened: graph-replay blocks of two
variants over an L2-cold pool, the record's structure, and a variant against
itself never deciding KEEP or REJECT."""
import pytest

from cudalab_b200.evaluator import paired as pr

pytestmark = pytest.mark.gpu


def test_paired_short_run_record():
    rec = pr.paired("int4gemv", "int4gemv_mma", "int4gemv_mma_w4", 2048, 2048, flags=7,
                    rounds=5, samples=40, launches=8, pool_size=16, check=False)
    assert rec["n_rounds"] == 5 and len(rec["rounds"]) == 5
    for r in rec["rounds"]:
        assert r["parent_us"] > 0 and r["candidate_us"] > 0
        assert r["blocks"]["parent"]["n_raw"] == 40
    assert rec["decision"]["decision"] in (pr.KEEP, pr.REJECT, pr.NEUTRAL, pr.UNSTABLE)
    assert rec["statistical_relation"] in (pr.FASTER, pr.SLOWER, pr.UNRESOLVED)
    assert 0.5 < rec["parent_median_us"] < 50


def test_paired_self_comparison_is_not_decisive():
    rec = pr.paired("qgemv", "qgemv_mma", "qgemv_mma", 2048, 2048, flags=7,
                    rounds=5, samples=40, launches=8, pool_size=16, check=False)
    assert rec["decision"]["decision"] in (pr.NEUTRAL, pr.UNSTABLE)
    assert 0.9 < rec["summary"]["median"] < 1.1
