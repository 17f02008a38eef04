"""Restated LoopSpec scheduler and greedy decision rules (oracle, test-only).

Follows sglang_recurrent/loopspec/pipeline.py:
  PipelineLane        :13-42
  PipelineResult      :45-56
  _descends_from      :85-97
  _prune_ancestry     :100-121
  PipelineSchedule    :124-251
  continue_pipelined  :254-423
and sglang_recurrent/loopspec/decisions.py:
  DecisionOutcome              :32-42
  GreedyDecisionPolicy.resolve :136-184
The data classes keep the reference's field names so traces can be compared
field by field.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any


@dataclass
class PipelineLane:
    stage: int
    index: int
    token: int
    state: int | None = None
    branch: int = 0
    parent_branch: int | None = None
    origin_stage: int | None = None
    first_token: int | None = None
    first_state: Any = None
    second_token: int | None = None
    second_state: Any = None


@dataclass(frozen=True)
class PipelineResult:
    state: int
    prediction: int
    proposed: bool = False
    proposal_state: Any = None
    accepted_stage: int | None = None
    proposal_action: str | None = None


@dataclass(frozen=True)
class DecisionOutcome:
    prediction: int
    proposed: bool = False
    proposal_state: Any = None
    accepted_stage: int | None = None
    proposal_action: str | None = None
    first_rejected: bool = False
    second_rejected: bool = False


def descends_from(branch, ancestor, parents):
    """pipeline.py:85-97: walk parent ids until ancestor or None."""
    while branch is not None and branch != ancestor:
        branch = parents.get(branch)
    return branch == ancestor


def prune_ancestry(lanes, root, parents):
    """pipeline.py:100-121: keep only live paths, re-rooted at `root`."""
    live = {root}
    for lane in lanes:
        b = lane.branch
        while b != root:
            if b is None or b not in parents:
                raise RuntimeError("pipeline branch escaped the selected ancestry")
            live.add(b)
            b = parents[b]
    return {b: (None if b == root else parents[b]) for b in live}


@dataclass(frozen=True)
class PipelineSchedule:
    """pipeline.py:124-251 (S stages, K step, optional X second step)."""

    stages: int
    step_size: int
    second_step: int | None = None

    def __post_init__(self):
        S, K, X = self.stages, self.step_size, self.second_step
        if not isinstance(S, int) or S <= 0:
            raise ValueError(f"stages S must be a positive integer, got {S}")
        if not isinstance(K, int) or not 1 <= K < S or S % K:
            raise ValueError(f"step_size K must be a positive divisor of S with K < S; got K={K}, S={S}")
        if X is not None and (not isinstance(X, int) or not 1 < X < S // K):
            raise ValueError(f"second_step X must satisfy 1 < X < S/K so K*X < S; got X={X}, S/K={S // K}")

    @property
    def depth(self):
        return self.stages // self.step_size

    @property
    def proposal_stage(self):
        return self.step_size - 1

    @property
    def second_stage(self):
        return None if self.second_step is None else self.step_size * self.second_step - 1

    @property
    def endpoint_kinds(self):
        kinds = {self.proposal_stage: "q1"}
        if self.second_stage is not None:
            kinds[self.second_stage] = "q2"
        kinds[self.stages - 1] = "final"
        return kinds

    @property
    def endpoint_stages(self):
        return tuple(sorted(self.endpoint_kinds))

    @property
    def row_birth_sizes(self):
        if self.second_step is None:
            return [1] * self.depth
        births = [1] * self.second_step
        for t in range(self.second_step, self.depth):
            births.append(births[t - 1] + births[t - self.second_step])
        return births

    @property
    def max_rows(self):
        return sum(self.row_birth_sizes)

    def request_pool_capacity(self, *, has_pre_attention=True, has_post_attention=True):
        births = self.row_birth_sizes
        births.append(1 if self.second_step is None
                      else births[-1] + births[self.depth - self.second_step])
        post_steps = [s // self.step_size + 1 for s in self.endpoint_stages]
        root_rows = self.stages + int(has_pre_attention) + int(has_post_attention) * len(post_steps)
        return 2 * root_rows + sum(
            births[self.depth + 1 - age]
            * (self.step_size * age + int(has_pre_attention)
               + int(has_post_attention) * sum(step <= age for step in post_steps))
            for age in range(1, self.depth + 1)
        )

    def role_max_batch_sizes(self):
        births = self.row_birth_sizes
        post_steps = {0, self.depth - 1}
        if self.second_step is not None:
            post_steps.add(self.second_step - 1)
        return {
            "pre": births[-1],
            "recurrent": sum(births),
            "post": sum(births[self.depth - 1 - step] for step in post_steps),
        }


def continue_pipelined(first_token, max_new_tokens, executor):
    """pipeline.py:254-423, statement for statement in behaviour."""
    if max_new_tokens <= 0:
        raise ValueError("a committed first token requires a positive budget")
    sch = executor.schedule
    q1_stage = sch.proposal_stage
    q2_stage = sch.second_stage
    proposal_stages = {q1_stage, q2_stage} - {None}
    stride = sch.step_size
    final_stage = sch.stages - 1
    max_rows = sch.max_rows
    committed = [first_token]
    if max_new_tokens == 1:
        executor.retain_branches(())
        return committed

    next_branch = 1
    parents = {0: None}
    lanes = [PipelineLane(stage=0, index=1, token=first_token)]
    while len(committed) < max_new_tokens:
        results = list(executor.forward(lanes))
        if len(results) != len(lanes):
            raise ValueError("executor must return one result per lane")
        following, children = [], []
        final = None
        accepted_stage = None
        for lane, res in zip(lanes, results):
            end_stage = lane.stage + stride - 1
            if end_stage == final_stage:
                if final is not None:
                    raise RuntimeError("multiple branches reached the final stage")
                final = (lane, res)
                continue
            lane.stage = end_stage + 1
            lane.state = res.state
            if end_stage in proposal_stages and res.proposed:
                if end_stage == q1_stage:
                    lane.first_token = res.prediction
                    lane.first_state = res.proposal_state
                elif res.proposal_action in ("residual", "argmax"):
                    lane.second_token = res.prediction
                    lane.second_state = res.proposal_state
                else:
                    raise RuntimeError("q2 proposal has no branch action")
                if lane.index + 1 < max_new_tokens:
                    children.append(PipelineLane(
                        stage=0, index=lane.index + 1, token=res.prediction,
                        branch=next_branch, parent_branch=lane.branch,
                        origin_stage=end_stage))
                    parents[next_branch] = lane.branch
                    next_branch += 1
            following.append(lane)
        following.extend(children)

        if final is not None:
            lane, res = final
            if lane.index != len(committed):
                raise RuntimeError("pipeline attempted to commit out of order")
            committed.append(res.prediction)
            if executor.should_stop(committed):
                executor.retain_branches(())
                return committed
            if lane.index + 1 < max_new_tokens:
                selected = next((c for c in following
                                 if c.parent_branch == lane.branch
                                 and c.token == res.prediction
                                 and c.origin_stage == res.accepted_stage), None)
                if selected is None:
                    selected = PipelineLane(
                        stage=0, index=lane.index + 1, token=res.prediction,
                        branch=next_branch, parent_branch=lane.branch,
                        origin_stage=final_stage)
                    parents[next_branch] = lane.branch
                    next_branch += 1
                    following.append(selected)
                accepted_stage = res.accepted_stage
                keep = selected.branch
                following = [c for c in following if descends_from(c.branch, keep, parents)]
                parents = prune_ancestry(following, keep, parents)
            else:
                following = []

        if len(following) > max_rows:
            raise RuntimeError("speculative tree exceeded branch row limit")
        lanes = following
        executor.retain_branches(tuple(lanes), accepted_stage)
        if not lanes and len(committed) < max_new_tokens:
            raise RuntimeError("pipeline drained before generation completed")
    return committed


def greedy_resolve(lane, endpoint_kind, decision, proposal_state, schedule):
    """decisions.py:136-184: greedy proposal / verification rules."""
    prediction = decision[0]
    proposed = endpoint_kind == "q1" or (endpoint_kind == "q2" and prediction != lane.first_token)
    accepted_stage = None
    first_rejected = second_rejected = False
    if endpoint_kind == "final" and lane.first_token is not None:
        first_rejected = prediction != lane.first_token
        if not first_rejected:
            accepted_stage = schedule.proposal_stage
        elif lane.second_token is not None:
            second_rejected = prediction != lane.second_token
            if not second_rejected:
                accepted_stage = schedule.second_stage
    return DecisionOutcome(
        prediction=prediction, proposed=proposed, proposal_state=proposal_state,
        accepted_stage=accepted_stage,
        proposal_action="argmax" if endpoint_kind == "q2" and proposed else None,
        first_rejected=first_rejected, second_rejected=second_rejected)


# executor.py:35-45
LOOPSPEC_METRICS = (
    "pipeline_cycles", "pre_rows", "recurrent_rows", "post_rows",
    "verified_proposals", "first_rejections", "second_verifications",
    "second_acceptances", "second_rejections",
)


def accept_length(stats, schedule):
    """experiment_tools/result_parser.py:196-223: S*T / cycles, k2 = S without q2."""
    T = stats["decode_tokens"]
    S = schedule.stages
    k1 = schedule.step_size
    k2 = S if schedule.second_step is None else schedule.step_size * schedule.second_step
    first_reject = stats["first_rejections"]
    final_reject = stats["second_rejections"] + (
        first_reject - stats["second_verifications"])
    cycles = T * k1 + first_reject * (k2 - k1) + final_reject * (S - k2)
    return S * T / cycles if cycles else 0.0
