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
