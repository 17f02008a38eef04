"""The engine's C++ scheduler loop (no GPU) against reference-scheduler traces."""

import gzip
import json
import os

import pytest

from scripted_executor import CASES, METRICS, _mix, hash_decision

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "pipeline_traces.json.gz")


def _golden():
    with gzip.open(GOLDEN, "rt") as f:
        return json.load(f)


@pytest.mark.parametrize("device_logic", [False, True], ids=["host", "device-loop"])
@pytest.mark.parametrize("idx", range(len(CASES)))
def test_native_scheduler_matches_reference_trace(idx, device_logic):
    """The host scheduler and the device loop's scheduler (compiled for the
    host) both reproduce the reference scheduler's traces exactly."""
    from loopspec_b200.simulate import simulate_pipeline
    gold = _golden()[idx]
    S, K, X, q1, q2, n, seed, vocab, stop = CASES[idx]
    first = _mix(seed, 0, 0, 9) % vocab

    def decide(index, token, kind):
        return hash_decision(seed, vocab, q1, q2, index, token, kind)

    ids, stats, trace = simulate_pipeline(S, K, X, first, n, decide, stop_token=stop,
                                          device_logic=device_logic)
    assert ids == gold["committed"]
    for name in METRICS:
        assert stats[name] == gold["metrics"][name], name
    assert stats["decode_tokens"] == max(len(ids) - 1, 0)
    gold_lanes = [c["lanes"] for c in gold["trace"] if "lanes" in c]
    got_lanes = [c["lanes"] for c in trace if "lanes" in c]
    assert got_lanes == gold_lanes
    gold_ret = [(c["retain"], c["accepted_stage"]) for c in gold["trace"] if "retain" in c]
    got_ret = [(c["retain"], c["accepted_stage"]) for c in trace if "retain" in c]
    assert got_ret == gold_ret


@pytest.mark.parametrize("bad", [(4, 4, 0), (4, 3, 0), (4, 1, 1), (4, 1, 4)])
def test_native_scheduler_rejects_invalid_schedule(bad):
    from loopspec_b200._lib import EngineError
    from loopspec_b200.simulate import simulate_pipeline
    with pytest.raises(EngineError):
        simulate_pipeline(*bad, 0, 8, lambda i, t, k: 0)
