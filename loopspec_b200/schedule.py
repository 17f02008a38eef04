"""LoopSpec schedule and the scheduler<->executor protocol types.

Same names, fields and validation as the reference
(sglang_recurrent/loopspec/pipeline.py:13-82 for PipelineLane / PipelineResult /
PipelineExecutor and :124-251 for PipelineSchedule), so an executor built on
this engine can be driven by the reference's own `continue_pipelined`.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Protocol, Sequence


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


class PipelineExecutor(Protocol):
    schedule: "PipelineSchedule"

    def should_stop(self, output_ids: Sequence[int]) -> bool: ...

    def forward(self, lanes: Sequence[PipelineLane]) -> Sequence[PipelineResult]: ...

    def retain_branches(self, lanes: Sequence[PipelineLane], accepted_stage: int | None = None) -> None: ...


@dataclass(frozen=True)
class PipelineSchedule:
    stages: int
    step_size: int
    second_step: int | None = None

    def __post_init__(self):
        S, K, X = self.stages, self.step_size, self.second_step
        if not isinstance(S, int) or S <= 0:
            raise ValueError(f"the recurrence count must be at least 1 (got S={S})")
        if not isinstance(K, int) or not 1 <= K < S or S % K:
            raise ValueError(f"--first must divide the recurrence count and be smaller than it (got K={K}, S={S})")
        if X is not None and (not isinstance(X, int) or not 1 < X < S // K):
            raise ValueError(f"--second must be a multiple of --first strictly between it and the recurrence count (got X={X}, S/K={S // K})")

    @property
    def depth(self) -> int:
        return self.stages // self.step_size

    @property
    def proposal_stage(self) -> int:
        return self.step_size - 1

    @property
    def second_stage(self) -> int | None:
        return None if self.second_step is None else self.step_size * self.second_step - 1

    @property
    def endpoint_kinds(self) -> dict[int, str]:
        kinds = {self.proposal_stage: "q1"}
        if self.second_stage is not None:
            kinds[self.second_stage] = "q2"
        kinds[self.stages - 1] = "final"
        return kinds

    @property
    def endpoint_stages(self) -> tuple[int, ...]:
        return tuple(sorted(self.endpoint_kinds))

    @property
    def row_birth_sizes(self) -> list[int]:
        if self.second_step is None:
            return [1] * self.depth
        births = [1] * self.second_step
        for t in range(self.second_step, self.depth):
            births.append(births[t - 1] + births[t - self.second_step])
        return births

    @property
    def max_rows(self) -> int:
        return sum(self.row_birth_sizes)

    def role_max_batch_sizes(self) -> dict[str, int]:
        births = self.row_birth_sizes
        post_steps = {0, self.depth - 1}
        if self.second_step is not None:
            post_steps.add(self.second_step - 1)
        return {"pre": births[-1], "recurrent": sum(births),
                "post": sum(births[self.depth - 1 - s] for s in post_steps)}


# Work/acceptance counters (executor.py:35-45).
LOOPSPEC_METRICS = (
    "pipeline_cycles", "pre_rows", "recurrent_rows", "post_rows",
    "verified_proposals", "first_rejections", "second_verifications",
    "second_acceptances", "second_rejections",
)


def accept_length(stats: dict, schedule: PipelineSchedule) -> float:
    """Mean accepted length S*T / cycles (experiment_tools/result_parser.py:196-223)."""
    T = stats["decode_tokens"]
    S = schedule.stages
    k1 = schedule.step_size
    k2 = S if schedule.second_step is None else schedule.step_size * schedule.second_step
    fr = stats["first_rejections"]
    final_reject = stats["second_rejections"] + fr - stats["second_verifications"]
    cycles = T * k1 + fr * (k2 - k1) + final_reject * (S - k2)
    return S * T / cycles if cycles else 0.0
