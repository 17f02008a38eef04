"""Scenario recipe shared by make_sampling_golden.py and the oracle's golden test.

A scenario is a short LoopSpec readout pipeline for one sampling setting: in
cycle t, lane t gets its q1 readout, lane t-1 its q2 readout (when the
schedule has q2) and lane t-2 (or t-1 without q2) its final readout, all rows
of one decision call, as the reference's SamplingDecisionPolicy sees them
(sampling/policy.py:220-283). The logits of lane n's readouts are its own
base row plus readout noise, so proposals are sometimes accepted and
sometimes rejected. Logits come from torch's CPU generator, so the test
recomputes them from the recipe instead of storing them.
"""

from __future__ import annotations

import torch

# (name, vocab, temperature, top_k, top_p, has_q2, logit scale, readout noise, cycles, seed)
SCENARIOS = [
    ("topp07_q2", 5000, 1.0, 0, 0.7, True, 2.0, 0.6, 14, 1),
    ("topp09_T07_q2", 4096, 0.7, 0, 0.9, True, 1.5, 0.8, 14, 2),
    ("full_q2", 2500, 1.0, 0, 1.0, True, 1.0, 0.5, 14, 3),
    ("joint_k50_p08_q2", 5000, 1.3, 50, 0.8, True, 2.0, 0.7, 14, 4),
    ("topp05_no_q2", 6200, 1.0, 0, 0.5, False, 2.5, 0.4, 12, 5),
    ("sharp_topp095_q2", 3000, 0.5, 0, 0.95, True, 3.0, 1.0, 14, 6),
]


def readout_logits(vocab, scale, noise, seed, lane, kind):
    """fp32 logits [vocab] of lane `lane`'s readout of `kind` (0 q1, 1 q2, 2 final)."""
    g = torch.Generator().manual_seed(1_000_003 * seed + 7919 * lane)
    base = torch.randn(vocab, generator=g) * scale
    g.manual_seed(1_000_003 * seed + 7919 * lane + 101 * (kind + 1))
    return (base + torch.randn(vocab, generator=g) * noise).float()


def cycle_rows(t, cycles, has_q2):
    """Readout rows of cycle t: list of (lane, kind), kind 0 q1 / 1 q2 / 2 final.

    Lane n reads out q1 in cycle n, q2 in cycle n + 1 (with q2) and its final
    readout one cycle after its last draft; every fourth lane has no draft
    and only a final readout, which then draws the token directly."""
    lag = 2 if has_q2 else 1
    rows = []
    for n in range(cycles - lag):
        direct = n % 4 == 3
        if not direct and t == n:
            rows.append((n, 0))
        if has_q2 and not direct and t == n + 1:
            rows.append((n, 1))
        if t == n + lag:
            rows.append((n, 2))
    return rows


KIND_NAMES = ("q1", "q2", "final")
