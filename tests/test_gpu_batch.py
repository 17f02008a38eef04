"""Several requests decoded together (ls_generate_batch) on the GPU.

Each request of a batch must commit exactly the tokens, and count exactly the
pipeline events, it commits and counts when served alone with the same seed:
the kernels compute every lane independently of the other lanes of a call, and
each request keeps its own timelines, state slots and random stream. Also runs
the tiny configuration as the benchmark plan states it (4 prompts of 32
uniform-random ids, 64 greedy tokens, LoopSpec 1:2 against autoregressive)
with per-token logits checked against the fp32 oracle (2e-2 max-abs).
"""

import pytest
import torch

from loopspec_b200._lib import EngineError
from loopspec_b200.executor import generate_autoregressive, generate_loopspec, generate_loopspec_batch
from oracle.executor import teacher_forced_logits

from test_gpu_engine import LOGIT_TOL, make, prompt_for

pytestmark = pytest.mark.gpu

COUNTERS = ("pipeline_cycles", "pre_rows", "recurrent_rows", "post_rows", "verified_proposals",
            "first_rejections", "second_verifications", "second_acceptances", "second_rejections",
            "decode_tokens")


def _prompts(cfg, lens, seed):
    return [prompt_for(cfg, n, seed=seed + i) for i, n in enumerate(lens)]


@pytest.mark.parametrize("name,K,X", [("tiny", 1, 2), ("tiny-raven-llama", 2, 2), ("tiny-raven-olmo", 1, 4)])
@pytest.mark.parametrize("mode", ["loopspec", "ar"])
def test_batched_greedy_requests_equal_their_batch1_runs(name, K, X, mode):
    cfg, eng, _ = make(name, K, X, max_requests=4)
    prompts = _prompts(cfg, [7, 33, 20, 1], seed=11)
    ids, per, total = eng.generate_batch(prompts, 24, mode=mode)
    for i, p in enumerate(prompts):
        alone, st = eng.generate(p, 24, mode=mode)
        assert ids[i] == alone, (i, mode)
        if mode == "loopspec":
            for k in COUNTERS:
                assert per[i][k] == st[k], (i, k)
    assert total["decode_tokens"] == sum(len(x) - 1 for x in ids)
    # the batch streams each core iteration's weights once for all requests
    if mode == "loopspec":
        assert total["core_calls"] < sum(p["pipeline_cycles"] for p in per) * eng.schedule.step_size
    eng.close()


def test_batched_sampled_requests_equal_their_batch1_runs():
    cfg, eng, _ = make("tiny", 1, 2, max_requests=3)
    prompts = _prompts(cfg, [12, 5, 30], seed=21)
    samp = {"temperature": 1.0, "top_k": 0, "top_p": 0.9}
    seeds = [101, 202, 303]
    ids, per, _ = generate_loopspec_batch(eng, prompts, 32, sampling=samp, seeds=seeds)
    for i, p in enumerate(prompts):
        alone, st = generate_loopspec(eng, p, 32, sampling=samp, seed=seeds[i])
        assert ids[i] == alone, i
        for k in COUNTERS:
            assert per[i][k] == st[k], (i, k)
    # the seed, not the batch position, selects the stream
    ids2, _, _ = generate_loopspec_batch(eng, prompts[::-1], 32, sampling=samp, seeds=seeds[::-1])
    assert ids2[::-1] == ids
    eng.close()


@pytest.mark.parametrize("mode", ["loopspec", "ar"])
def test_mixed_greedy_and_sampled_requests_equal_their_batch1_runs(mode):
    """Per-request sampling parameters (ls_generate_batch_sampling): greedy and
    sampled requests share the batch's calls; each commits what it commits
    alone with its own parameters and seed."""
    cfg, eng, _ = make("tiny", 1, 2, max_requests=4)
    prompts = _prompts(cfg, [9, 25, 14, 3], seed=31)
    samp = [None, {"temperature": 1.0, "top_k": 0, "top_p": 0.9}, None,
            {"temperature": 0.8, "top_k": 40, "top_p": 1.0}]
    seeds = [7, 8, 9, 10]
    ids, per, _ = generate_loopspec_batch(eng, prompts, 24, sampling=samp, seeds=seeds, mode=mode)
    alone_fn = generate_loopspec if mode == "loopspec" else generate_autoregressive
    for i, p in enumerate(prompts):
        alone, st = alone_fn(eng, p, 24, sampling=samp[i], seed=seeds[i])
        assert ids[i] == alone, (i, mode)
        if mode == "loopspec":
            for k in COUNTERS:
                assert per[i][k] == st[k], (i, k)
    # greedy requests of the batch took the argmax: they equal AR-greedy alone
    g0, _ = generate_autoregressive(eng, prompts[0], 24)
    assert ids[0] == g0
    eng.close()


def test_more_requests_than_configured_are_refused():
    cfg, eng, _ = make("tiny", 1, 2, max_requests=2)
    with pytest.raises(EngineError):
        eng.generate_batch(_prompts(cfg, [4, 4, 4], seed=1), 8)
    ids, _ = eng.generate(prompt_for(cfg, 6), 8)      # still usable
    assert len(ids) == 8
    eng.close()


def test_baseline_config1_four_prompts_64_greedy_tokens():
    """tiny Ouro-style model, seed-0 init, 4 prompts of 32
    uniform-random ids (seed 0), 64 greedy tokens, LoopSpec 1:2 vs AR."""
    cfg, eng, om = make("tiny", 1, 2, max_requests=4)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab, (32,), generator=g).tolist() for _ in range(4)]
    ls, per, total = eng.generate_batch(prompts, 64, mode="loopspec")
    ar, _, _ = eng.generate_batch(prompts, 64, mode="ar")
    assert ls == ar
    assert all(len(x) == 64 for x in ls)
    assert total["decode_tokens"] == 4 * 63
    sch = eng.schedule
    for p, ids in zip(prompts, ls):
        # per-token final-depth logits of the committed path vs the fp32 oracle
        # position P - 1 + i (fed ids[i - 1], or the last prompt token) decides ids[i]
        P = len(p)
        tf = teacher_forced_logits(om, sch, p + ids[:-1], P - 1)
        worst = 0.0
        for i in range(len(ids)):
            lg = tf[(P - 1 + i, sch.stages - 1)].numpy()
            # the committed token is the argmax of the oracle's logits up to the tolerance
            worst = max(worst, float(lg.max() - lg[ids[i]]))
        assert worst <= 2 * LOGIT_TOL, worst
    eng.close()
