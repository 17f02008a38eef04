"""Pin the oracle's restated scheduler against traces of the reference scheduler."""

import gzip
import json
import os

import pytest

from conftest import REFERENCE_ROOT, reference_available
from oracle import pipeline as op
from scripted_executor import CASES, run_case

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "pipeline_traces.json.gz")


def _golden():
    with gzip.open(GOLDEN, "rt") as f:
        return json.load(f)


def _oracle_run(case):
    return run_case(case, op.continue_pipelined, op.PipelineSchedule,
                    op.PipelineResult, op.greedy_resolve)


@pytest.mark.parametrize("idx", range(len(CASES)))
def test_oracle_scheduler_matches_reference_trace(idx):
    gold = _golden()[idx]
    got = json.loads(json.dumps(_oracle_run(CASES[idx])))
    assert got["case"] == gold["case"]
    assert got["committed"] == gold["committed"]
    assert got["metrics"] == gold["metrics"]
    assert got["trace"] == gold["trace"]
    assert got["max_rows"] == gold["max_rows"]
    assert got["request_pool_capacity"] == gold["request_pool_capacity"]
    assert got["role_max_batch_sizes"] == gold["role_max_batch_sizes"]


def test_schedule_shapes_match_survey_table():
    # (S, K, X) -> (max_rows, role max batch pre/recurrent/post, request rows)
    table = {
        (4, 1, None): (4, (1, 4, 2), 33),
        (4, 1, 2): (7, (3, 7, 6), 66),
        (32, 2, None): (16, (1, 16, 2), 375),
        (32, 2, 4): (249, (69, 249, 96), 3314),
        (32, 2, 5): (139, (34, 139, 46), 1929),
        (32, 4, 2): (54, (21, 54, 35), 1148),
    }
    for (S, K, X), (rows, (p, r, q), req) in table.items():
        s = op.PipelineSchedule(S, K, X)
        assert s.max_rows == rows
        assert s.role_max_batch_sizes() == {"pre": p, "recurrent": r, "post": q}
        assert s.request_pool_capacity() == req


@pytest.mark.parametrize("bad", [(4, 4, None), (4, 3, None), (4, 0, None), (4, 1, 1), (4, 1, 4), (32, 2, 16)])
def test_schedule_rejects_invalid(bad):
    with pytest.raises(ValueError):
        op.PipelineSchedule(*bad)


def test_budget_validation():
    class Ex:
        schedule = op.PipelineSchedule(4, 1, 2)
    with pytest.raises(ValueError):
        op.continue_pipelined(0, 0, Ex())


@pytest.mark.skipif(not reference_available(), reason="reference tree not mounted")
def test_live_reference_equals_oracle():
    import sys
    sys.path.insert(0, REFERENCE_ROOT)
    from sglang_recurrent.loopspec import decisions, pipeline
    resolve = lambda *a: decisions.GreedyDecisionPolicy.resolve(None, *a)  # noqa: E731
    for case in CASES:
        ref = run_case(case, pipeline.continue_pipelined, pipeline.PipelineSchedule,
                       pipeline.PipelineResult, resolve)
        got = _oracle_run(case)
        assert ref["committed"] == got["committed"]
        assert ref["trace"] == got["trace"]
        assert ref["metrics"] == got["metrics"]
