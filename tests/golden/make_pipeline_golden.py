"""Record scheduler golden traces by running the REFERENCE scheduler unmodified.

Loads sglang_recurrent/loopspec/pipeline.py (continue_pipelined,
PipelineSchedule, PipelineResult) and decisions.py
(GreedyDecisionPolicy.resolve) from the reference tree and drives them with
ScriptedExecutor over every case in scripted_executor.CASES. Output:
pipeline_traces.json.gz beside this script. Run here (where the reference tree is
mounted):  python tests/golden/make_pipeline_golden.py [reference_root]
"""

from __future__ import annotations

import gzip
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from scripted_executor import CASES, run_case  # noqa: E402


def load_reference(root):
    sys.path.insert(0, root)
    from sglang_recurrent.loopspec import decisions, pipeline  # noqa: WPS433
    resolve = decisions.GreedyDecisionPolicy.resolve

    def resolve_fn(lane, kind, decision, state, schedule):
        return resolve(None, lane, kind, decision, state, schedule)

    return pipeline, resolve_fn


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LOOPSPEC_REFERENCE", "/root/reference")
    pipeline, resolve = load_reference(root)
    traces = [run_case(c, pipeline.continue_pipelined, pipeline.PipelineSchedule,
                       pipeline.PipelineResult, resolve) for c in CASES]
    path = os.path.join(HERE, "pipeline_traces.json.gz")
    with gzip.open(path, "wt") as f:
        json.dump(traces, f, separators=(",", ":"))
    print(f"wrote {len(traces)} traces to {path}")


if __name__ == "__main__":
    main()
