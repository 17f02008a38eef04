"""generation_metrics records: pinned against lines the reference's
log_decode_metrics produced (tests/golden/metrics_records.json, made by
tests/golden/make_metrics_golden.py), and the request-level interval rule."""

import json
import logging
import os

from loopspec_b200.metrics import decode_metrics, format_record, log_decode_metrics, request_metrics

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "metrics_records.json")


def test_records_match_the_reference_lines():
    cases = json.load(open(GOLDEN))
    assert len(cases) >= 6
    for c in cases:
        assert format_record(decode_metrics(c["decode_tokens"], c["decode_seconds"], c["stats"])) == c["line"]


def test_logger_emits_the_record(caplog):
    log = logging.getLogger("ls_metrics_test")
    with caplog.at_level(logging.INFO, logger="ls_metrics_test"):
        log_decode_metrics(log, 3, 1.5, None)
    assert caplog.records[-1].getMessage() == 'generation_metrics {"decode_seconds":1.5,"decode_tok_s":2.0,"decode_tokens":3}'


def test_request_interval_excludes_the_first_token():
    st = {"pipeline_cycles": 10, "verified_proposals": 4, "first_rejections": 1, "second_verifications": 1,
          "second_acceptances": 1, "second_rejections": 0, "decode_host_s": 0.5}
    m = request_metrics([5, 6, 7, 8, 9], st)
    assert (m["decode_tokens"], m["decode_seconds"], m["decode_tok_s"]) == (4, 0.5, 8.0)
    assert (m["first_accept"], m["first_reject"], m["second_skip"]) == (3, 1, 0)
    one = request_metrics([5], st)
    assert (one["decode_tokens"], one["decode_seconds"], one["decode_tok_s"]) == (0, 0.0, None)
    assert "pipeline_cycles" not in request_metrics([5, 6], st, loopspec=False)


def test_validity_rule_matches_the_reference_parser():
    from loopspec_b200.metrics import record_valid
    cases = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "metrics_validity.json")))
    assert any(c["valid"] for c in cases) and any(not c["valid"] for c in cases)
    for c in cases:
        assert record_valid(c["record"]) == c["valid"], c["record"]


def test_native_scheduler_counters_pass_the_reference_log_checks():
    # Every scripted schedule case (stops, rejections at both stages, early
    # EOS): the record of its committed output satisfies the parser's rules.
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    from scripted_executor import CASES, _mix, hash_decision
    from loopspec_b200.metrics import decode_metrics, record_valid
    from loopspec_b200.simulate import simulate_pipeline
    for S, K, X, q1, q2, n, seed, vocab, stop in CASES:
        first = _mix(seed, 0, 0, 9) % vocab
        ids, stats, _ = simulate_pipeline(
            S, K, X, first, n, lambda i, t, k: hash_decision(seed, vocab, q1, q2, i, t, k), stop_token=stop)
        rec = decode_metrics(max(len(ids) - 1, 0), 1.0, {k: int(v) for k, v in stats.items()
                                                          if not isinstance(v, float)})
        assert record_valid(rec), (S, K, X, q1, q2, n, seed, stop, rec)
