"""Record generation_metrics lines from the REFERENCE's log_decode_metrics.

Loads sglang_recurrent/server/metrics.py from the reference tree by file path
(it imports only json and logging), calls log_decode_metrics for every case
below with a capturing logger, and writes the (inputs, line) pairs to
metrics_records.json beside this script. Run here (where the reference tree is
mounted):  python tests/golden/make_metrics_golden.py [reference_root]
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
    print(f"wrote {len(out)} records")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
