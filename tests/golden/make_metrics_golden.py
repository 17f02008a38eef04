"""Record generation_metrics lines from the REFERENCE's log_decode_metrics,
and the reference result parser's verdict on a set of records.

Loads sglang_recurrent/server/metrics.py and experiment_tools/result_parser.py
from the reference tree by file path (both import only the standard library).
Calls log_decode_metrics for every case below with a capturing logger and
writes the (inputs, line) pairs to metrics_records.json. Asks
GenerationMetrics._valid about every record of VALIDITY (valid ones and ones
that break each rule) and writes (record, verdict) pairs to
metrics_validity.json. Run here (where the reference tree is mounted):
python tests/golden/make_metrics_golden.py [reference_root]
"""

from __future__ import annotations

import importlib.util
import json
import logging
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

_STATS = {"pipeline_cycles": 12276, "verified_proposals": 3069, "first_rejections": 3069,
          "second_verifications": 3069, "second_acceptances": 0, "second_rejections": 3069}
CASES = [
    (1023, 4.71, _STATS),
    (0, 0.0, _STATS),
    (5, 0.0, {"pipeline_cycles": 9, "verified_proposals": 4, "first_rejections": 1,
              "second_verifications": 0, "second_acceptances": 0, "second_rejections": 0}),
    (127, 3.4491, {"pipeline_cycles": 2020, "verified_proposals": 127, "first_rejections": 127,
                   "second_verifications": 127, "second_acceptances": 1, "second_rejections": 126}),
    (64, 0.25, None),
    (0, 1.5, None),
]


_OK = {"decode_seconds": 2.0, "decode_tokens": 10, "decode_tok_s": 5.0, "pipeline_cycles": 40,
       "first_accept": 4, "first_reject": 6, "second_skip": 1, "second_accept": 2, "second_reject": 3}
VALIDITY = [
    _OK,
    {"decode_seconds": 0.0, "decode_tokens": 0, "decode_tok_s": None},
    {"decode_seconds": 1.5, "decode_tokens": 3, "decode_tok_s": 2.0},
    dict(_OK, decode_tokens=11),                    # tokens != first_accept + first_reject
    dict(_OK, second_skip=2),                       # second fields do not add up
    dict(_OK, first_accept=-1, decode_tokens=5),    # negative field
    dict(_OK, decode_seconds=float("inf")),
    dict(_OK, decode_seconds=-1.0),
    dict(_OK, decode_tokens=10.0),                  # float token count
    dict(_OK, decode_seconds=True),
    {k: v for k, v in _OK.items() if k != "second_reject"},   # partial rejection fields
    {"decode_seconds": 1.0},
    [1, 2],
]


class _Capture(logging.Handler):
    def __init__(self):
        super().__init__()
        self.lines = []

    def emit(self, record):
        self.lines.append(record.getMessage())


def main(root):
    spec = importlib.util.spec_from_file_location(
        "ref_metrics", os.path.join(root, "sglang_recurrent", "server", "metrics.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    log = logging.getLogger("ref_metrics_capture")
    log.setLevel(logging.INFO)
    cap = _Capture()
    log.addHandler(cap)
    out = []
    for tokens, seconds, stats in CASES:
        mod.log_decode_metrics(log, tokens, seconds, stats)
        out.append({"decode_tokens": tokens, "decode_seconds": seconds, "stats": stats,
                    "line": cap.lines[-1]})
    with open(os.path.join(HERE, "metrics_records.json"), "w") as f:
        json.dump(out, f, indent=1)
    spec = importlib.util.spec_from_file_location(
        "ref_result_parser", os.path.join(root, "experiment_tools", "result_parser.py"))
    parser = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(parser)
    verdicts = [{"record": r, "valid": bool(parser.GenerationMetrics._valid(r))} for r in VALIDITY]
    with open(os.path.join(HERE, "metrics_validity.json"), "w") as f:
        json.dump(verdicts, f, indent=1)
    print(f"wrote {len(out)} records and {len(verdicts)} verdicts")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LOOPSPEC_REFERENCE", "/root/reference"))
