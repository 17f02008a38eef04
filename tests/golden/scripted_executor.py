"""A deterministic PipelineExecutor with a hash "model", for scheduler traces.

Used by make_pipeline_golden.py (driving the reference scheduler) and by the
tests (driving the oracle restatement and the engine's native scheduler), so
all of them see identical decisions. The final-depth token for a lane depends
only on (index, input token); q1/q2 drafts agree with it at tunable rates.
State slots follow the reference's _StateSlotPool rule
(sglang_recurrent/loopspec/executor.py:76-107), metric counting follows
executor.py:268-281.
"""

from __future__ import annotations

import heapq

METRICS = ("pipeline_cycles", "pre_rows", "recurrent_rows", "post_rows",
           "verified_proposals", "first_rejections", "second_verifications",
           "second_acceptances", "second_rejections")


def _mix(*xs):
    h = 0x9E3779B97F4A7C15
    for x in xs:
        h ^= (x + 0x632BE59BD9B4E019 + (h << 6) + (h >> 2)) & 0xFFFFFFFFFFFFFFFF
        h = (h * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        h ^= h >> 31
    return h


def hash_decision(seed, vocab, q1_rate, q2_rate, index, token, kind):
    """Token predicted at a readout of the lane (index, input token)."""
    final = _mix(seed, index, token, 0) % vocab
    if kind == "final":
        return final
    r = (_mix(seed, index, token, 1) % 10_000) / 10_000.0
    if kind == "q1":
        return final if r < q1_rate else _mix(seed, index, token, 2) % vocab
    q1 = hash_decision(seed, vocab, q1_rate, q2_rate, index, token, "q1")
    if q1 == final:
        return q1
    r2 = (_mix(seed, index, token, 4) % 10_000) / 10_000.0
    return final if r2 < q2_rate else _mix(seed, index, token, 3) % vocab


class ScriptedExecutor:
    def __init__(self, schedule, resolve, *, seed, vocab, q1_rate, q2_rate,
                 stop_token=None):
        self.schedule = schedule
        self.resolve = resolve
        self.seed, self.vocab = seed, vocab
        self.q1_rate, self.q2_rate = q1_rate, q2_rate
        self.stop_token = stop_token
        self.kinds = schedule.endpoint_kinds
        self._free = list(range(schedule.max_rows))
        self._live = set()
        self.metrics = dict.fromkeys(METRICS, 0)
        self.trace = []

    def should_stop(self, ids):
        return self.stop_token is not None and ids[-1] == self.stop_token

    def _acquire(self):
        if not self._free:
            raise RuntimeError("state slots exhausted")
        s = heapq.heappop(self._free)
        self._live.add(s)
        return s

    def forward(self, lanes):
        sch = self.schedule
        K = sch.step_size
        slots = [l.state if l.state is not None else self._acquire() for l in lanes]
        cycle = {"lanes": [[l.stage, l.index, l.token, l.branch,
                            -1 if l.parent_branch is None else l.parent_branch,
                            -1 if l.origin_stage is None else l.origin_stage,
                            slots[i]] for i, l in enumerate(lanes)],
                 "decisions": []}
        ends = [l.stage + K - 1 for l in lanes]
        endpoints = {i: self.kinds[e] for i, e in enumerate(ends) if e in self.kinds}
        self.metrics["pipeline_cycles"] += 1
        self.metrics["pre_rows"] += sum(l.stage == 0 for l in lanes)
        self.metrics["recurrent_rows"] += len(lanes) * K
        self.metrics["post_rows"] += len(endpoints)
        results = []
        for i, l in enumerate(lanes):
            kind = endpoints.get(i)
            if kind is None:
                results.append(self._result(slots[i], 0))
                continue
            tok = hash_decision(self.seed, self.vocab, self.q1_rate, self.q2_rate,
                                l.index, l.token, kind)
            cycle["decisions"].append([i, tok])
            o = self.resolve(l, kind, [tok], None, sch)
            if kind == "final":
                m = self.metrics
                m["verified_proposals"] += 1
                sv = o.first_rejected and l.second_token is not None
                m["first_rejections"] += o.first_rejected
                m["second_verifications"] += sv
                m["second_acceptances"] += sv and o.accepted_stage == sch.second_stage
                m["second_rejections"] += sv and o.second_rejected
            results.append(self._result(slots[i], o.prediction, o.proposed,
                                        o.accepted_stage, o.proposal_action))
        self.trace.append(cycle)
        return results

    def _result(self, state, prediction, proposed=False, accepted_stage=None, action=None):
        return self.result_cls(state=state, prediction=prediction, proposed=proposed,
                               proposal_state=None, accepted_stage=accepted_stage,
                               proposal_action=action)

    def retain_branches(self, lanes, accepted_stage=None):
        keep = {l.state for l in lanes if l.state is not None}
        released = self._live - keep
        self._live &= keep
        for s in released:
            heapq.heappush(self._free, s)
        self.trace.append({"retain": sorted([l.branch, -1 if l.parent_branch is None else l.parent_branch]
                                            for l in lanes),
                           "accepted_stage": -1 if accepted_stage is None else accepted_stage})


# (S, K, X, q1_rate, q2_rate, max_new_tokens, seed, vocab, stop_token)
CASES = [
    (4, 1, None, 0.0, 0.0, 40, 1, 64, None),
    (4, 1, None, 0.7, 0.0, 60, 2, 64, None),
    (4, 1, 2, 0.0, 0.0, 40, 3, 64, None),
    (4, 1, 2, 0.5, 0.5, 80, 4, 64, None),
    (4, 1, 2, 0.9, 0.9, 80, 5, 16, None),
    (4, 1, 2, 1.0, 1.0, 50, 6, 64, None),
    (4, 2, None, 0.6, 0.0, 50, 7, 64, None),
    (32, 2, None, 0.5, 0.0, 60, 8, 64, None),
    (32, 2, 4, 0.4, 0.6, 70, 9, 64, None),
    (32, 2, 5, 0.5, 0.5, 60, 10, 64, None),
    (32, 4, 2, 0.3, 0.8, 60, 11, 32, None),
    (32, 2, 4, 0.8, 0.8, 60, 12, 8, 3),
    (4, 1, 2, 0.5, 0.5, 1, 13, 64, None),
    (4, 1, 2, 0.5, 0.5, 2, 14, 64, None),
    (8, 2, 2, 0.5, 0.5, 45, 15, 64, 7),
]


def run_case(case, continue_pipelined, schedule_cls, result_cls, resolve):
    S, K, X, q1, q2, n, seed, vocab, stop = case
    sch = schedule_cls(S, K, X)
    ex = ScriptedExecutor(sch, resolve, seed=seed, vocab=vocab, q1_rate=q1,
                          q2_rate=q2, stop_token=stop)
    ex.result_cls = result_cls
    first = _mix(seed, 0, 0, 9) % vocab
    out = continue_pipelined(first, n, ex)
    return {"case": list(case), "first": first, "committed": out,
            "metrics": ex.metrics, "trace": ex.trace,
            "max_rows": sch.max_rows,
            "request_pool_capacity": sch.request_pool_capacity(),
            "role_max_batch_sizes": sch.role_max_batch_sizes()}
