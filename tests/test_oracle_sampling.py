"""Checks of the oracle's sampling restatement (CPU)."""

import numpy as np
import pytest
import torch

from oracle import sampling as S


def ref_filter_torch(logits, T, top_p):
    """The reference's top-p-only path (distributions.py:44-70) in fp32 torch."""
    probs = torch.softmax(torch.tensor(logits, dtype=torch.float32)[None] / T, dim=-1)
    sp = probs.sort(dim=-1, descending=True).values
    cum = sp.cumsum(dim=-1)
    th = torch.full((1, 1), top_p, dtype=torch.float32)
    idx = torch.searchsorted(cum, th, right=False).clamp_max_(probs.shape[-1] - 1)
    cut = sp.gather(-1, idx)
    f = torch.where(probs >= cut, probs, 0)
    return (f / f.sum(dim=-1, keepdim=True))[0].double().numpy()


@pytest.mark.parametrize("seed,V,T,top_p", [(0, 4096, 1.0, 0.7), (1, 5000, 0.7, 0.9), (2, 300, 1.3, 0.5)])
def test_top_p_filter_matches_reference_algorithm(seed, V, T, top_p):
    rng = np.random.default_rng(seed)
    logits = rng.normal(0, 2.0, V)
    got = S.filtered(logits, T, 0, top_p)
    ref = ref_filter_torch(logits, T, top_p)
    assert ((got > 0) == (ref > 0)).mean() > 0.999       # same support up to fp32 boundary ties
    assert np.abs(got - ref).max() < 1e-6


def test_top_k_and_joint_filters():
    p = S.softmax(np.log(np.array([0.4, 0.3, 0.2, 0.1])), 1.0)
    f = S.filtered(np.log(p), 1.0, 2, 1.0)
    assert np.allclose(f, [0.4 / 0.7, 0.3 / 0.7, 0, 0])
    f = S.filtered(np.log(p), 1.0, 3, 0.5)               # top-p keeps 2, top-k 3 -> intersection 2
    assert np.allclose(f, [0.4 / 0.7, 0.3 / 0.7, 0, 0])
    ties = np.log(np.array([0.25, 0.25, 0.25, 0.25]))
    assert np.allclose(S.filtered(ties, 1.0, 0, 0.3), 0.25)   # boundary ties are kept


def test_pick_known_answers():
    one_hot = np.zeros(5000)
    one_hot[0] = 1
    assert S.pick(one_hot, 0.999) == 0                    # sampler.py warmup: one-hot -> 0
    one_hot[:] = 0
    one_hot[4097] = 3.0
    assert S.pick(one_hot, 0.5) == 4097
    w = np.ones(4100)
    assert S.pick(w, 0.0) == 0 and S.pick(w, 0.99999) == 4099
    assert S.pick(w, 2048.5 / 4100) == 2048               # chunk boundary


def test_verify_accepts_equal_distributions():
    p = S.softmax(np.arange(10.0), 1.0)
    d, *_ = S.decide("final", np.log(p), q1=p, first=3, u=(0.9999, 0.5, 0.5))
    assert d == [3, 0, 1, 0, 0]                           # p == q -> always accept


def test_uniforms_are_in_unit_interval_and_keyed():
    a = S.uniforms(7, 3, 1)
    assert all(0.0 <= x < 1.0 for x in a)
    assert a == S.uniforms(7, 3, 1) and a != S.uniforms(7, 4, 1) and a != S.uniforms(8, 3, 1)


@pytest.mark.parametrize("with_q2", [False, True])
def test_speculative_decision_is_lossless(with_q2):
    """The committed token is distributed as the final readout P (chi-square)."""
    rng = np.random.default_rng(11 + with_q2)
    V = 6
    lg_q1, lg_q2, lg_p = (rng.normal(0, 1.2, V) for _ in range(3))
    Q1 = S.filtered(lg_q1, 1.0, 0, 1.0)
    D2 = S.filtered(lg_q2, 1.0, 0, 1.0)
    P = S.filtered(lg_p, 1.0, 0, 1.0)
    n = 40000
    counts = np.zeros(V)
    for _ in range(n):
        u = rng.random(6)
        x = S.pick(Q1, u[0])
        second = R = None
        if with_q2:
            d2, _, _, R_ = S.decide("q2", lg_q2, q1=Q1, first=x, u=(u[1], 0, 0))
            if d2[1]:
                second, R = d2[0], R_
        d, *_ = S.decide("final", lg_p, q1=Q1, r=R, first=x, second=second, u=(u[2], u[3], u[4]))
        counts[d[0]] += 1
    expected = P * n
    chi2 = ((counts - expected) ** 2 / expected).sum()
    assert chi2 < 25.0, (chi2, counts / n, P)            # 5 dof: p ~ 1e-4 at 25


def test_no_residual_mass_edge_cases():
    p = S.softmax(np.array([2.0, 1.0, 0.5, -1.0]), 1.0)
    # q2 identical to q1: no residual mass -> no second proposal, the q1 token stands
    d, _, _, R = S.decide("q2", np.log(p), q1=p, first=1, u=(0.3, 0, 0))
    assert d == [1, 0, 0, 0, 0] and not R.any()
    # R equal to F: max(F - R, 0) has no mass, and the q2 token is accepted with
    # probability F[y] / R[y] = 1 (the fallback to F is reached only through rounding)
    q1 = np.array([0.1, 0.6, 0.2, 0.1])
    P = S.filtered(np.log(p), 1.0, 0, 1.0)
    F = np.maximum(P - q1, 0)
    F /= F.sum()
    info = {}
    d, *_ = S.decide("final", np.log(p), q1=q1, r=F.copy(), first=1, second=0,
                     u=(0.9999, 0.99999, 0.5), info=info)
    assert info["mG"] == 0.0
    assert d == [0, 0, 2, 1, 0]
