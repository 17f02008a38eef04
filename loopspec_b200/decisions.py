"""Greedy proposal / verification rules (sglang_recurrent/loopspec/decisions.py:32-184).

The engine computes the argmax on the GPU (lowest index on ties, like
torch.argmax); these host rules turn one endpoint's token into a proposal or a
final verification outcome, exactly as the reference's GreedyDecisionPolicy.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any


@dataclass(frozen=True, slots=True)
class DecisionOutcome:
    prediction: int
    proposed: bool = False
    proposal_state: Any = None
    accepted_stage: int | None = None
    proposal_action: str | None = None
    first_rejected: bool = False
    second_rejected: bool = False


class GreedyDecisionPolicy:
    def resolve(self, lane, endpoint_kind, decision, proposal_state, schedule) -> DecisionOutcome:
        """q1 always proposes; q2 proposes iff it differs from q1; final accepts q1, else q2."""
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
