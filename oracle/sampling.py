"""float64 restatement of the LoopSpec sampling decisions (oracle, test-only).

Follows the reference:
  filtered_probabilities            sampling/distributions.py:14-86
      softmax(logits / T) in fp32; top-p keeps every probability >= the first
      sorted value whose cumulative mass reaches top_p (ties kept); top-k keeps
      >= the k-th largest; both -> the larger cutoff; renormalise.
  categorical pick (chunk = 2048)   sampling/sampler.py:49-102
      target = u * total; first chunk whose inclusive CDF exceeds target, then
      first token in it whose inclusive CDF exceeds target - preceding mass.
  q2 conditional residual           sampler.py:178-344 and policy.py:78-111
      r = max(q2 - q1, 0) with r[x] = 0 for the q1 token x; draw y ~ r;
      R = r / sum(r); action = sum(r) > 0 and q2[x] < q1[x].
  final verification                sampler.py:428-460, policy.py:144-195
      accept x if u < min(1, P[x] / Q1[x]).
  rejection fallback                sampling/rejection.py:42-97
      F = norm(max(P - Q1, 0)) (or norm(P) if no mass); with a q2 token y and
      its R: accept y if u1 < min(1, F[y] / R[y]); otherwise sample
      norm(max(F - R, 0)) (or F if no mass / no q2) with u2.
  decision rows                     policy.py:197-218, 255-283
      (token, proposed, accepted_code, q1_rejected, q2_rejected).
  resolve                           policy.py:285-308

Uniforms are the engine's choice (the reference draws torch.rand on the
device RNG, which no other implementation can reproduce): word k of
Philox4x32-10(counter = (cycle, row, 0, 0), key = (seed low, seed high)),
u_k = (word >> 8) * 2^-24, with u0 for the row's draw or verification, u1 for
the q2 test and u2 for the fallback draw after a q1 rejection.
"""

from __future__ import annotations

import numpy as np

from .model import philox4x32
from .pipeline import DecisionOutcome

CHUNK = 2048


def uniforms(seed, cycle, row):
    ctr = np.array([[cycle, row, 0, 0]], dtype=np.uint64)
    w = philox4x32(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))[0]
    return [float(int(x) >> 8) * (1.0 / (1 << 24)) for x in w[:3]]


def softmax(logits, temperature):
    x = np.asarray(logits, dtype=np.float64) / float(temperature)
    e = np.exp(x - x.max())
    return e / e.sum()


def _cutoff_top_p(p, top_p):
    s = np.sort(p)[::-1]
    c = np.cumsum(s)
    i = int(np.searchsorted(c, top_p, side="left"))
    return s[min(i, len(s) - 1)]


def filtered(logits, temperature, top_k, top_p):
    p = softmax(logits, temperature)
    V = len(p)
    k = 0 if top_k >= V else top_k
    if k == 0 and top_p >= 1:
        return p
    cut = 0.0
    if top_p < 1:
        cut = _cutoff_top_p(p, top_p)
    if k:
        cut = max(cut, np.sort(p)[::-1][k - 1])
    f = np.where(p >= cut, p, 0.0)
    return f / f.sum()


def pick(w, u):
    """Inverse-CDF pick with the reference's chunking; w need not be normalised."""
    w = np.asarray(w, dtype=np.float64)
    V = len(w)
    nch = (V + CHUNK - 1) // CHUNK
    sums = np.array([w[i * CHUNK:(i + 1) * CHUNK].sum() for i in range(nch)])
    target = u * sums.sum()
    cdf = np.cumsum(sums)
    hits = np.nonzero(cdf > target)[0]
    ch = int(hits[0]) if len(hits) else 0
    pre = sums[:ch].sum()
    seg = np.cumsum(w[ch * CHUNK:(ch + 1) * CHUNK])
    hits = np.nonzero(seg > target - pre)[0]
    return ch * CHUNK + (int(hits[0]) if len(hits) else 0)


def decide(kind, logits, *, q1=None, r=None, first=None, second=None, temperature=1.0,
           top_k=0, top_p=1.0, u=(0.0, 0.0, 0.0), info=None):
    """One endpoint row. Returns (decision5, P, new_q1, new_r).

    `info` (optional dict) receives the residual masses of a rejection
    fallback: "mG" = sum max(F - R, 0). When it is tiny, F and R nearly
    coincide and the fallback's support is decided by rounding, so fp32 and
    float64 implementations may legitimately draw different tokens there.
    """
    P = filtered(logits, temperature, top_k, top_p)
    if kind == "q1":
        x = pick(P, u[0])
        return [x, 1, 0, 0, 0], P, P, None
    if kind == "q2":
        x = first
        res = np.maximum(P - q1, 0.0)
        res[x] = 0.0
        mass = res.sum()
        y = pick(res, u[0])
        R = res / mass if mass > 0 else np.zeros_like(res)
        action = int(mass > 0 and P[x] < q1[x])
        return [y if action else x, action, action, 0, 0], P, None, R
    if first is None:
        return [pick(P, u[0]), 0, 0, 0, 0], P, None, None
    x = first
    if u[0] < min(1.0, P[x] / q1[x]):
        return [x, 0, 1, 0, 0], P, None, None
    F = np.maximum(P - q1, 0.0)
    mF = F.sum()
    F = F / mF if mF > 0 else P / P.sum()
    has2 = second is not None
    acc2 = False
    fallback = F
    if has2:
        y = second
        acc2 = bool(u[1] < min(1.0, F[y] / r[y]))
        G = np.maximum(F - r, 0.0)
        mG = G.sum()
        if info is not None:
            info["mG"] = float(mG)
        if mG > 0:
            fallback = G / mG
    s = pick(fallback, u[2])
    token = second if acc2 else s
    return [token, 0, 2 if acc2 else 0, 1, int(has2 and not acc2)], P, None, None


def sampling_resolve(lane, endpoint_kind, decision, proposal_state, schedule):
    """policy.py:285-308."""
    prediction, proposed, code, q1_rej, q2_rej = decision
    proposed = bool(proposed)
    stage = schedule.proposal_stage if code == 1 else schedule.second_stage if code == 2 else None
    return DecisionOutcome(
        prediction=prediction, proposed=proposed,
        proposal_state=proposal_state if proposed else None,
        accepted_stage=stage,
        proposal_action="residual" if endpoint_kind == "q2" and proposed else None,
        first_rejected=bool(q1_rej), second_rejected=bool(q2_rej))
