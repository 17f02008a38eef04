"""Oracle PipelineExecutor and AR generation over OracleModel (test-only).

Restates, for one request at batch 1:
  LosslessLoopSpecExecutor (sglang_recurrent/loopspec/executor.py:110-397):
    _StateSlotPool :76-107, _prepare_cycle :205-237, forward :293-367,
    _make_pipeline_result :239-290 (metric counting), retain_branches :369-389
  RecurrentRequest.prefill (loopspec/request.py:111-192): every prompt token
    through pre, all S core depths and each post endpoint with attention.
  BranchManager timeline semantics (loopspec/branching/manager.py:207-232,
    357-388): a branch's missing (role, depth) timeline forks the parent's
    timeline of the same role/depth, sharing its current prefix.
  LoopedRecurrentServingModel (modeling/serving.py:185-239): AR = pre, S core
    iterations each on its own timeline, post.
Physical cleanup (row/slot release) has no effect on results, so this oracle
never frees a timeline; branch ids are never reused within one generation.
"""

from __future__ import annotations

import heapq

import torch

from .model import Timeline
from .pipeline import (
    LOOPSPEC_METRICS, PipelineLane, PipelineResult, PipelineSchedule,
    continue_pipelined, greedy_resolve,
)


def argmax_first(logits):
    """torch.argmax semantics: lowest index among maxima."""
    return int(torch.argmax(logits).item())


class _Node:
    def __init__(self, parent):
        self.parent = parent
        self.timelines = {}


class StateSlotPool:
    """executor.py:76-107: lowest free slot first; retain releases the rest."""

    def __init__(self, capacity):
        self.capacity = capacity
        self._free = list(range(capacity))
        self._live = set()

    def acquire(self):
        if not self._free:
            raise RuntimeError(
                "pipeline requires more recurrent state slots than configured "
                f"(max_rows={self.capacity})")
        s = heapq.heappop(self._free)
        self._live.add(s)
        return s

    def retain(self, slots):
        keep = set(slots)
        released = self._live - keep
        self._live &= keep
        for s in released:
            heapq.heappush(self._free, s)


class OracleLoopSpecExecutor:
    def __init__(self, model, schedule, prompt_ids, max_new_tokens, *,
                 should_stop=None, record=None):
        if not prompt_ids:
            raise ValueError("the prompt must contain at least one token")
        self.model = model
        self.schedule = schedule
        self.endpoint_kind = schedule.endpoint_kinds
        self.prompt = list(prompt_ids)
        self.prefill_len = len(self.prompt) - 1
        self.max_new_tokens = max_new_tokens
        self._stop = should_stop or (lambda ids: False)
        self.metrics = dict.fromkeys(LOOPSPEC_METRICS, 0)
        self.slots = StateSlotPool(schedule.max_rows)
        self.state = {}
        self.record = record
        cfg = model.cfg
        self.has_pre_attn = cfg["n_pre_layers"] > 0
        self.has_post_attn = cfg["n_post_layers"] > 0
        self.nodes = {0: _Node(None)}
        self.first_logits = self._prefill()
        self._first = argmax_first(self.first_logits)

    def _n_layers(self, role):
        c = self.model.cfg
        return {"pre": c["n_pre_layers"], "core": c["n_core_layers"], "post": c["n_post_layers"]}[role]

    def _prefill(self):
        root = self.nodes[0].timelines
        m = self.model
        S = self.schedule.stages
        if self.has_pre_attn:
            root[("pre", 0)] = Timeline(self._n_layers("pre"))
        for s in range(S):
            root[("core", s)] = Timeline(self._n_layers("core"))
        if self.has_post_attn:
            for e in self.schedule.endpoint_stages:
                root[("post", e)] = Timeline(self._n_layers("post"))
        logits = None
        for pos, tok in enumerate(self.prompt):
            h, inj = m.pre(tok, pos, root.get(("pre", 0)))
            saved = {}
            for s in range(S):
                h = m.core(h, inj, pos, root[("core", s)])
                if s in self.endpoint_kind:
                    saved[s] = h
            if self.has_post_attn:
                for e in self.schedule.endpoint_stages:
                    out = m.post(saved[e], pos, root[("post", e)])
                    if e == S - 1:
                        logits = out
            else:
                logits = m.post(h, pos, None)
        return logits

    def first_token(self):
        return self._first

    def should_stop(self, ids):
        return self._stop(ids)

    def _node(self, branch, parent):
        n = self.nodes.get(branch)
        if n is None:
            p = self.nodes.get(parent)
            if p is None:
                raise RuntimeError(f"branch {branch} has unavailable parent {parent}")
            n = _Node(p)
            self.nodes[branch] = n
        return n

    def _timeline(self, node, role, depth):
        key = (role, depth)
        tl = node.timelines.get(key)
        if tl is None:
            tl = node.parent.timelines[key].fork()
            node.timelines[key] = tl
        return tl

    def forward(self, lanes):
        sch = self.schedule
        K = sch.step_size
        m = self.model
        starts = [l.stage for l in lanes]
        ends = [s + K - 1 for s in starts]
        slots = [l.state if l.state is not None else self.slots.acquire() for l in lanes]
        pre_rows = [i for i, l in enumerate(lanes) if l.stage == 0]
        endpoints = {i: self.endpoint_kind[e] for i, e in enumerate(ends) if e in self.endpoint_kind}
        nodes = [self._node(l.branch, l.parent_branch) for l in lanes]
        pos = [self.prefill_len + l.index for l in lanes]
        for i in pre_rows:
            tl = self._timeline(nodes[i], "pre", 0) if self.has_pre_attn else None
            self.state[slots[i]] = m.pre(lanes[i].token, pos[i], tl)
        for off in range(K):
            for i, l in enumerate(lanes):
                h, inj = self.state[slots[i]]
                tl = self._timeline(nodes[i], "core", starts[i] + off)
                self.state[slots[i]] = (m.core(h, inj, pos[i], tl), inj)
        decisions = {}
        for i in endpoints:
            tl = self._timeline(nodes[i], "post", ends[i]) if self.has_post_attn else None
            logits = m.post(self.state[slots[i]][0], pos[i], tl)
            decisions[i] = [argmax_first(logits)]
            if self.record is not None:
                self.record.append((lanes[i].index, ends[i], logits))
        self.metrics["pipeline_cycles"] += 1
        self.metrics["pre_rows"] += len(pre_rows)
        self.metrics["recurrent_rows"] += len(lanes) * K
        self.metrics["post_rows"] += len(endpoints)
        out = []
        for i, l in enumerate(lanes):
            kind = endpoints.get(i)
            if kind is None:
                out.append(PipelineResult(state=slots[i], prediction=0))
                continue
            o = greedy_resolve(l, kind, decisions[i], None, sch)
            if kind == "final":
                self.metrics["verified_proposals"] += 1
                second_verified = o.first_rejected and l.second_token is not None
                self.metrics["first_rejections"] += o.first_rejected
                self.metrics["second_verifications"] += second_verified
                self.metrics["second_acceptances"] += (
                    second_verified and o.accepted_stage == sch.second_stage)
                self.metrics["second_rejections"] += second_verified and o.second_rejected
            out.append(PipelineResult(
                state=slots[i], prediction=o.prediction, proposed=o.proposed,
                proposal_state=None, accepted_stage=o.accepted_stage,
                proposal_action=o.proposal_action))
        return out

    def retain_branches(self, lanes, accepted_stage=None):
        self.slots.retain(l.state for l in lanes if l.state is not None)
        for l in sorted(lanes, key=lambda x: x.branch):
            if l.branch and l.branch not in self.nodes:
                self._node(l.branch, l.parent_branch)


def generate_loopspec_oracle(model, schedule, prompt_ids, max_new_tokens, *,
                             should_stop=None, record=None):
    """executor.py:400-458 minus timing: returns (ids, stats)."""
    ex = OracleLoopSpecExecutor(model, schedule, prompt_ids, max_new_tokens,
                                should_stop=should_stop, record=record)
    first = ex.first_token()
    out = [first]
    if not ex.should_stop(out):
        out = continue_pipelined(first, max_new_tokens, ex)
    stats = dict(ex.metrics)
    stats["decode_tokens"] = max(len(out) - 1, 0)
    return out, stats


def generate_ar_oracle(model, stages, prompt_ids, max_new_tokens, *,
                       should_stop=None, record=None):
    """serving.py:216-239 one token at a time: pre, S core iterations, post."""
    stop = should_stop or (lambda ids: False)
    cfg = model.cfg
    tl_pre = Timeline(cfg["n_pre_layers"]) if cfg["n_pre_layers"] else None
    tl_core = [Timeline(cfg["n_core_layers"]) for _ in range(stages)]
    tl_post = Timeline(cfg["n_post_layers"]) if cfg["n_post_layers"] else None
    seq = list(prompt_ids)
    out = []
    pos = 0
    while True:
        tok = seq[pos]
        h, inj = model.pre(tok, pos, tl_pre)
        for s in range(stages):
            h = model.core(h, inj, pos, tl_core[s])
        logits = model.post(h, pos, tl_post)
        pos += 1
        if pos < len(prompt_ids):
            continue
        if record is not None:
            record.append((len(out), stages - 1, logits))
        nxt = argmax_first(logits)
        out.append(nxt)
        seq.append(nxt)
        if len(out) >= max_new_tokens or stop(out):
            return out


def teacher_forced_logits(model, schedule, tokens, start):
    """Logits of every readout depth at positions >= start for a fixed token path.

    tokens = prompt + committed completion; position p feeds tokens[p]. For
    post roles with attention each endpoint depth has its own timeline, as in
    LoopSpec (request.py:157-176). Returns {(position, end_stage): logits}.
    """
    cfg = model.cfg
    S = schedule.stages
    ends = schedule.endpoint_stages
    tl_pre = Timeline(cfg["n_pre_layers"]) if cfg["n_pre_layers"] else None
    tl_core = [Timeline(cfg["n_core_layers"]) for _ in range(S)]
    tl_post = {e: Timeline(cfg["n_post_layers"]) for e in ends} if cfg["n_post_layers"] else None
    out = {}
    for pos, tok in enumerate(tokens):
        h, inj = model.pre(tok, pos, tl_pre)
        for s in range(S):
            h = model.core(h, inj, pos, tl_core[s])
            if s in ends and (tl_post is not None or pos >= start):
                lg = model.post(h, pos, tl_post[s] if tl_post is not None else None)
                if pos >= start:
                    out[(pos, s)] = lg
    return out


__all__ = [
    "OracleLoopSpecExecutor", "StateSlotPool", "PipelineSchedule", "PipelineLane",
    "generate_loopspec_oracle", "generate_ar_oracle", "argmax_first",
]
