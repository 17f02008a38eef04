"""Request-level entry points over the engine, mirroring the reference API.

* `B200Executor` implements the reference's PipelineExecutor protocol
  (sglang_recurrent/loopspec/pipeline.py:59-82) the way
  LosslessLoopSpecExecutor does (loopspec/executor.py:110-397): it prefills
  in its constructor, keeps the state-slot pool and the counters on the host,
  and runs each cycle (pre / K core / post + decisions) as one `ls_cycle`
  call on the GPU. Any `continue_pipelined` -- the reference's own included --
  can drive it; this is the engine's parity mode. Greedy decisions resolve
  with GreedyDecisionPolicy.resolve (decisions.py:136-184), sampled ones with
  SamplingDecisionPolicy.resolve (sampling/policy.py:285-308).
* `generate_loopspec` has the reference signature (executor.py:400-423) and
  runs the whole request inside the engine (`ls_generate`): prefill, first
  token and the native scheduler loop, with no Python per cycle.
* `generate_autoregressive` is the unrolled baseline (serving.py:216-239).
* `generate_loopspec_batch` serves several requests together
  (`ls_generate_batch`); each commits what it commits alone. The reference
  serves LoopSpec one request at a time (server/cli.py:88-89).
"""

from __future__ import annotations

import heapq
from typing import Callable, Sequence

from .decisions import DecisionOutcome, GreedyDecisionPolicy
from .engine import Engine
from .schedule import LOOPSPEC_METRICS, PipelineLane, PipelineResult


class _StateSlotPool:
    """Lowest free bank row first (executor.py:76-107)."""

    def __init__(self, capacity):
        self.capacity = capacity
        self._free = list(range(capacity))
        self._live = set()

    def acquire(self):
        if not self._free:
            raise RuntimeError("pipeline requires more recurrent state slots than "
                               f"configured (max_rows={self.capacity})")
        s = heapq.heappop(self._free)
        self._live.add(s)
        return s

    def retain(self, slots):
        keep = set(slots)
        released = self._live - keep
        self._live &= keep
        for s in released:
            heapq.heappush(self._free, s)


def sampling_resolve(lane, endpoint_kind, decision, proposal_state, schedule):
    """Interpret one (token, proposed, accepted_code, q1_rej, q2_rej) row (policy.py:285-308)."""
    prediction, proposed, code, q1_rej, q2_rej = decision
    proposed = bool(proposed)
    stage = schedule.proposal_stage if code == 1 else schedule.second_stage if code == 2 else None
    return DecisionOutcome(
        prediction=prediction, proposed=proposed,
        proposal_state=proposal_state if proposed else None, accepted_stage=stage,
        proposal_action="residual" if endpoint_kind == "q2" and proposed else None,
        first_rejected=bool(q1_rej), second_rejected=bool(q2_rej))


def _seed_of(generator, seed):
    if seed is not None:
        return int(seed)
    if generator is not None:
        return int(generator.initial_seed())
    return 0


def apply_sampling(engine: Engine, sampling, generator=None, seed=None):
    """Set greedy (sampling None) or {temperature, top_k, top_p} for the next request."""
    if sampling is None:
        engine.set_sampling(0.0, 1, 1.0, 0)
    else:
        engine.set_sampling(float(sampling.get("temperature", 1.0)), int(sampling.get("top_k", 0)),
                            float(sampling.get("top_p", 1.0)), _seed_of(generator, seed))


class B200Executor:
    """PipelineExecutor for one request on a B200 engine."""

    def __init__(self, engine: Engine, prompt_ids: Sequence[int], max_new_tokens: int, *,
                 sampling=None, generator=None, seed=None,
                 should_stop: Callable[[Sequence[int]], bool] | None = None,
                 record_logits: bool = False):
        if not prompt_ids:
            raise ValueError("the prompt must contain at least one token")
        self.engine = engine
        self.schedule = engine.schedule
        self.endpoint_kind = self.schedule.endpoint_kinds
        apply_sampling(engine, sampling, generator, seed)
        self.sampled = engine.sampling
        self.resolve = sampling_resolve if self.sampled else GreedyDecisionPolicy().resolve
        self._slots = _StateSlotPool(self.schedule.max_rows)
        self._should_stop = should_stop or (lambda ids: False)
        self.metrics = dict.fromkeys(LOOPSPEC_METRICS, 0)
        self.record_logits = record_logits
        self.logits_log = []        # (index, end_stage, logits) per readout
        self.decision_log = []      # (cycle, row, kind, state slot, first, second, decision)
        self.cycles = 0
        self._first = engine.prefill(list(prompt_ids))

    def first_token(self):
        return self._first

    def should_stop(self, ids):
        return self._should_stop(ids)

    def finish_without_pipeline(self):
        self.engine.retain([])

    def forward(self, lanes: Sequence[PipelineLane]) -> list[PipelineResult]:
        sch = self.schedule
        K = sch.step_size
        slots = [l.state if l.state is not None else self._slots.acquire() for l in lanes]
        rows = [[l.stage, l.index, l.token, l.branch,
                 -1 if l.parent_branch is None else l.parent_branch, slots[i],
                 -1 if l.first_token is None else l.first_token,
                 -1 if l.second_token is None else l.second_token]
                for i, l in enumerate(lanes)]
        if self.record_logits:
            dec, logits = self.engine.cycle(rows, want_logits=True)
        else:
            dec, logits = self.engine.cycle(rows), None
        self.cycles += 1
        ends = [l.stage + K - 1 for l in lanes]
        endpoints = {i: self.endpoint_kind[e] for i, e in enumerate(ends) if e in self.endpoint_kind}
        m = self.metrics
        m["pipeline_cycles"] += 1
        m["pre_rows"] += sum(l.stage == 0 for l in lanes)
        m["recurrent_rows"] += len(lanes) * K
        m["post_rows"] += len(endpoints)
        out = []
        for row, (i, kind) in enumerate(endpoints.items()):
            self.decision_log.append((self.cycles, row, kind, slots[i], rows[i][6], rows[i][7],
                                      [int(v) for v in dec[i]]))
        for i, l in enumerate(lanes):
            kind = endpoints.get(i)
            if kind is None:
                out.append(PipelineResult(state=slots[i], prediction=0))
                continue
            if logits is not None:
                self.logits_log.append((l.index, ends[i], logits[i].copy()))
            d = [int(v) for v in dec[i]]
            o = self.resolve(l, kind, d if self.sampled else [d[0]], None, sch)
            if kind == "final":
                m["verified_proposals"] += 1
                sv = o.first_rejected and l.second_token is not None
                m["first_rejections"] += o.first_rejected
                m["second_verifications"] += sv
                m["second_acceptances"] += sv and o.accepted_stage == sch.second_stage
                m["second_rejections"] += sv and o.second_rejected
            out.append(PipelineResult(state=slots[i], prediction=o.prediction, proposed=o.proposed,
                                      proposal_state=None, accepted_stage=o.accepted_stage,
                                      proposal_action=o.proposal_action))
        return out

    def retain_branches(self, lanes: Sequence[PipelineLane], accepted_stage=None) -> None:
        self._slots.retain(l.state for l in lanes if l.state is not None)
        self.engine.retain([(l.branch, l.parent_branch) for l in lanes])

    def stats(self):
        return dict(self.metrics)


def generate_loopspec(runner: Engine, prompt_ids: Sequence[int], max_new_tokens: int, *,
                      sampling=None, generator=None, should_stop=None, stop_token=None, seed=None):
    """Generate completion ids for one prompt; returns (ids, stats).

    Same meaning as the reference's generate_loopspec: sampling None means
    greedy, else {temperature, top_k, top_p} with `generator` (or `seed`)
    fixing the random stream; ids exclude the prompt and uncommitted drafts;
    stats hold the executor counters and decode_tokens (excluding the first
    token), plus decode timing. `stop_token` ends generation when committed
    (EOS); `should_stop(ids)` sees the whole committed output after every
    commit and ends generation when it returns True (pipeline.py:64).
    """
    if max_new_tokens <= 0:
        raise ValueError("a committed first token requires a positive budget")
    apply_sampling(runner, sampling, generator, seed)
    return runner.generate(list(prompt_ids), max_new_tokens, mode="loopspec", stop_token=stop_token,
                           should_stop=should_stop)


def generate_autoregressive(runner: Engine, prompt_ids: Sequence[int], max_new_tokens: int, *,
                            sampling=None, generator=None, stop_token=None, seed=None):
    """Plain decoding: every token runs pre, all S core iterations, post."""
    apply_sampling(runner, sampling, generator, seed)
    return runner.generate(list(prompt_ids), max_new_tokens, mode="ar", stop_token=stop_token)


def generate_loopspec_batch(runner: Engine, prompts: Sequence[Sequence[int]], max_new_tokens: int, *,
                            sampling=None, seeds=None, stop_token=None, mode="loopspec"):
    """Generate for several prompts together; returns (ids per request,
    stats per request, batch stats). `sampling` applies to every request, or
    is a list with one entry per request (None = greedy), so greedy and
    sampled requests share a batch; request i draws from seeds[i] (default:
    0, 1, 2, ...), so it commits what generate_loopspec(..., sampling=its
    entry, seed=seeds[i]) commits for it alone."""
    if max_new_tokens <= 0:
        raise ValueError("a committed first token requires a positive budget")
    if seeds is None:
        seeds = list(range(len(prompts)))
    if isinstance(sampling, (list, tuple)):
        return runner.generate_batch([list(p) for p in prompts], max_new_tokens, mode=mode,
                                     stop_token=stop_token, seeds=seeds, sampling=list(sampling))
    apply_sampling(runner, sampling, None, seeds[0] if seeds else 0)
    return runner.generate_batch([list(p) for p in prompts], max_new_tokens, mode=mode,
                                 stop_token=stop_token, seeds=seeds)
