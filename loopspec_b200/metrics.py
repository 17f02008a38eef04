"""The `generation_metrics` record the reference's schedulers log per request.

Restates sglang_recurrent/server/metrics.py:8-50 (log_decode_metrics): one
log line "generation_metrics <json>" with compact separators and sorted keys,
holding decode_seconds, decode_tokens and decode_tok_s (null without tokens
or time) and, for LoopSpec requests, the executor counters pipeline_cycles,
first_accept, first_reject, second_skip, second_accept, second_reject. The
reference's offline result parser locates records by that prefix, so the
engine's requests can feed the same experiment tooling.

The decode interval follows loopspec_scheduler.py:364-375: it starts after the
first completion token and excludes it, so decode_tokens = outputs - 1, and a
request with at most one output token logs (0, 0.0).
"""

from __future__ import annotations

import json
import math
from logging import Logger
from typing import Mapping

PREFIX = "generation_metrics"


def decode_metrics(decode_tokens: int, decode_seconds: float,
                   loopspec_stats: Mapping[str, int] | None = None) -> dict:
    """The record's fields (metrics.py:22-43)."""
    m: dict = {
        "decode_seconds": decode_seconds,
        "decode_tokens": decode_tokens,
        "decode_tok_s": decode_tokens / decode_seconds if decode_tokens and decode_seconds > 0 else None,
    }
    if loopspec_stats is not None:
        s = loopspec_stats
        m.update(
            pipeline_cycles=s["pipeline_cycles"],
            first_accept=s["verified_proposals"] - s["first_rejections"],
            first_reject=s["first_rejections"],
            second_skip=s["first_rejections"] - s["second_verifications"],
            second_accept=s["second_acceptances"],
            second_reject=s["second_rejections"],
        )
    return m


def format_record(metrics: Mapping) -> str:
    """The logged line (metrics.py:46-50)."""
    return f"{PREFIX} " + json.dumps(metrics, separators=(",", ":"), sort_keys=True)


def request_metrics(output_ids, stats: Mapping, loopspec: bool = True) -> dict:
    """Fields for one finished request from the engine's generate() stats:
    decode_host_s is the host time from the first token's commit to the end."""
    n = len(output_ids)
    counters = {k: int(stats[k]) for k in ("pipeline_cycles", "verified_proposals", "first_rejections",
                                           "second_verifications", "second_acceptances",
                                           "second_rejections")} if loopspec else None
    if n <= 1 or not stats.get("decode_host_s"):
        return decode_metrics(0, 0.0, counters)
    return decode_metrics(n - 1, float(stats["decode_host_s"]), counters)


def log_decode_metrics(logger: Logger, decode_tokens: int, decode_seconds: float,
                       loopspec_stats: Mapping[str, int] | None = None) -> None:
    """Emit one record, as the reference's function of the same name."""
    logger.info("%s", format_record(decode_metrics(decode_tokens, decode_seconds, loopspec_stats)))


def record_valid(m) -> bool:
    """The reference's acceptance rule for a record (experiment_tools/
    result_parser.py:102-141): non-negative int decode_tokens and finite
    non-negative decode_seconds; if any rejection field is present, all five
    are non-negative ints with decode_tokens == first_accept + first_reject and
    second_skip + second_accept + second_reject == first_reject."""
    if not isinstance(m, dict):
        return False
    t, sec = m.get("decode_tokens"), m.get("decode_seconds")
    if not (type(t) is int and t >= 0 and isinstance(sec, (int, float)) and not isinstance(sec, bool)
            and math.isfinite(sec) and sec >= 0):
        return False
    fields = ("first_accept", "first_reject", "second_skip", "second_accept", "second_reject")
    vals = [m.get(f) for f in fields]
    if any(v is not None for v in vals):
        if not all(type(v) is int and v >= 0 for v in vals):
            return False
        if t != m["first_accept"] + m["first_reject"] or \
                m["second_skip"] + m["second_accept"] + m["second_reject"] != m["first_reject"]:
            return False
    return True
