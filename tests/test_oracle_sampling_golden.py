"""The oracle's sampling decisions against the reference's own sampler (CPU).

tests/golden/sampling_golden.json holds every decision row that the
reference's SamplingDecisionPolicy (sampling/policy.py:220-283, with
sampler.py, rejection.py and distributions.py) produced over six readout
scenarios, with the uniforms it drew (tests/golden/make_sampling_golden.py).
Replaying each row through oracle.sampling.decide with the same logits and
uniforms must give the same integer row: token, proposed flag, accepted code,
q1 rejected, q2 rejected. The engine's GPU sampler is checked against this
oracle decision by decision (tests/test_gpu_sampling.py), so it inherits the pin.
"""

import json
import os

import pytest

from oracle import sampling as S
from sampling_cases import SCENARIOS, readout_logits

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sampling_golden.json")


def _scenarios():
    with open(GOLDEN) as f:
        return json.load(f)["scenarios"]


def test_fixture_matches_the_scenario_recipe():
    got = [(s["name"], s["vocab"], s["temperature"], s["top_k"], s["top_p"], s["has_q2"],
            s["scale"], s["noise"], s["cycles"], s["seed"]) for s in _scenarios()]
    assert got == [tuple(sc) for sc in SCENARIOS]


def _assign_uniforms(rows, lanes_before, decisions, draws):
    """Uniform tuples per row in the reference's draw order (policy.py:78-195,
    255-283): q2 residual draws, q1 draws, direct final draws, verification
    draws, then two per rejected verification (q2 test, fallback draw)."""
    kinds = [k for _, k in rows]
    q2 = [i for i, k in enumerate(kinds) if k == 1]
    q1 = [i for i, k in enumerate(kinds) if k == 0]
    direct = [i for i, k in enumerate(kinds) if k == 2 and lanes_before[i][0] is None]
    verify = [i for i, k in enumerate(kinds) if k == 2 and lanes_before[i][0] is not None]
    u = {i: [0.0, 0.0, 0.0] for i in range(len(rows))}
    d = iter(draws)
    for group in (q2, q1, direct, verify):
        if group:
            vals = next(d)
            assert len(vals) == len(group)
            for i, v in zip(group, vals):
                u[i][0] = v
    rejected = [i for i in verify if decisions[i][3] == 1]
    for i in rejected:
        vals = next(d)
        u[i][1], u[i][2] = vals
    assert next(d, None) is None
    return u


@pytest.mark.parametrize("sc", _scenarios(), ids=lambda s: s["name"])
def test_oracle_decisions_equal_the_reference_sampler(sc):
    V, T, top_k, top_p = sc["vocab"], sc["temperature"], sc["top_k"], sc["top_p"]
    lanes = {}
    n_rows = 0
    for call in sc["calls"]:
        rows = call["rows"]
        u = _assign_uniforms(rows, call["lanes_before"], call["decisions"], call["draws"])
        for i, (n, k) in enumerate(rows):
            ln = lanes.setdefault(n, {"x": None, "q1": None, "y": None, "r": None})
            assert (ln["x"], ln["y"]) == tuple(call["lanes_before"][i])
            logits = readout_logits(V, sc["scale"], sc["noise"], sc["seed"], n, k).double().numpy()
            kind = ("q1", "q2", "final")[k]
            dec, P, new_q1, new_r = S.decide(kind, logits, q1=ln["q1"], r=ln["r"], first=ln["x"],
                                             second=ln["y"], temperature=T, top_k=top_k,
                                             top_p=top_p, u=tuple(u[i]))
            assert dec == call["decisions"][i], (call["t"], n, kind)
            if k == 0:
                ln["x"], ln["q1"] = dec[0], new_q1
            elif k == 1 and dec[1]:
                ln["y"], ln["r"] = dec[0], new_r
            n_rows += 1
    assert n_rows == sum(len(c["rows"]) for c in sc["calls"])


def test_fixture_covers_every_decision_branch():
    seen = set()
    for sc in _scenarios():
        for call in sc["calls"]:
            for (n, k), dec, before in zip(call["rows"], call["decisions"], call["lanes_before"]):
                if k == 0:
                    seen.add("q1 draw")
                elif k == 1:
                    seen.add("q2 proposes" if dec[1] else "q2 declines")
                elif before[0] is None:
                    seen.add("direct final draw")
                elif dec[2] == 1:
                    seen.add("q1 accepted")
                elif dec[2] == 2:
                    seen.add("q2 accepted")
                elif dec[4]:
                    seen.add("both rejected, fallback")
                else:
                    seen.add("q1 rejected without q2, fallback")
    assert seen == {"q1 draw", "q2 proposes", "q2 declines", "direct final draw", "q1 accepted",
                    "q2 accepted", "both rejected, fallback", "q1 rejected without q2, fallback"}


def test_a_planted_mistake_in_the_oracle_is_caught():
    """Swapping the rejection fallback's two uniforms (q2 test and fallback
    draw) in the replay must break at least one golden row: the fixture
    discriminates the draw order, not only the shapes."""
    mismatches = 0
    for sc in _scenarios():
        V, T, top_k, top_p = sc["vocab"], sc["temperature"], sc["top_k"], sc["top_p"]
        lanes = {}
        for call in sc["calls"]:
            u = _assign_uniforms(call["rows"], call["lanes_before"], call["decisions"], call["draws"])
            for i, (n, k) in enumerate(call["rows"]):
                ln = lanes.setdefault(n, {"x": None, "q1": None, "y": None, "r": None})
                ln["x"], ln["y"] = call["lanes_before"][i]
                logits = readout_logits(V, sc["scale"], sc["noise"], sc["seed"], n, k).double().numpy()
                wrong = (u[i][0], u[i][2], u[i][1])
                dec, _, new_q1, new_r = S.decide(("q1", "q2", "final")[k], logits, q1=ln["q1"], r=ln["r"],
                                                 first=ln["x"], second=ln["y"], temperature=T,
                                                 top_k=top_k, top_p=top_p, u=wrong)
                mismatches += dec != call["decisions"][i]
                if k == 0:
                    ln["q1"] = new_q1
                elif k == 1 and dec[1]:
                    ln["r"] = new_r
    assert mismatches > 0
