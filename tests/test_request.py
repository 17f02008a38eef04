"""Request semantics (loopspec_b200.request) against the reference scheduler's
rules (server/loopspec_scheduler.py:49-148 and :288-375), on a fake engine so
no GPU is needed: which options abort, what runs the model, how greedy and
seeded sampling are selected, and the finish reasons."""

import pytest

from loopspec_b200.request import run_request, unsupported_options


class FakeEngine:
    def __init__(self, out):
        self.out, self.calls, self.sampling_calls = out, [], []

    def set_sampling(self, temperature=0.0, top_k=0, top_p=1.0, seed=0):
        self.sampling_calls.append((temperature, top_k, top_p, seed))

    def generate(self, ids, max_new, *, mode, stop_token=None, should_stop=None):
        self.calls.append((list(ids), max_new, mode, stop_token))
        out = list(self.out[:max_new])
        if stop_token is not None and stop_token in out:
            out = out[: out.index(stop_token) + 1]
        if should_stop is not None:   # one commit per token
            for i in range(1, len(out) + 1):
                if should_stop(out[:i]):
                    out = out[:i]
                    break
        stats = {"pipeline_cycles": 2 * len(out), "verified_proposals": len(out), "first_rejections": 1,
                 "second_verifications": 1, "second_acceptances": 0, "second_rejections": 1,
                 "decode_tokens": len(out) - 1, "decode_host_s": 0.25}
        return out, stats


def test_supported_requests_list_nothing():
    assert unsupported_options({"input_ids": [1], "sampling_params": {"max_new_tokens": 4}}) == []
    assert unsupported_options({"input_ids": [1], "stream": True,
                                "sampling_params": {"stream_interval": 1, "top_p": 0.7}}) == []


@pytest.mark.parametrize("field,value,label", [
    ("mm_inputs", {"images": [1]}, "multimodal input"),
    ("lora_id", "a", "LoRA"),
    ("bootstrap_room", 3, "distributed request routing"),
    ("return_logprob", True, "return_logprob"),
    ("input_embeds", [[0.0]], "input_embeds"),
    ("require_reasoning", True, "hybrid reasoning"),
])
def test_request_features_abort(field, value, label):
    eng = FakeEngine([5, 6])
    r = run_request(eng, {"input_ids": [1, 2], field: value, "sampling_params": {"max_new_tokens": 2}})
    assert r["finish_reason"] == "abort" and label in r["message"] and not eng.calls


@pytest.mark.parametrize("params,label", [
    ({"regex": "a+"}, "constrained decoding"), ({"min_p": 0.1}, "min_p"),
    ({"min_new_tokens": 2}, "min_new_tokens"), ({"max_new_tokens": None}, "unbounded max_new_tokens"),
    ({"repetition_penalty": 1.1}, "sampling penalties"), ({"logit_bias": {"3": 1.0}}, "logit_bias"),
])
def test_sampling_features_abort(params, label):
    assert label in unsupported_options({"input_ids": [1], "sampling_params": params})


def test_stream_interval_and_order():
    r = {"input_ids": [1], "stream": True, "lora_id": "x",
         "sampling_params": {"stream_interval": 4, "min_p": 0.2}}
    assert unsupported_options(r) == ["LoRA", "min_p", "stream_interval other than 1"]


def test_empty_prompt_and_zero_budget_do_no_model_work():
    eng = FakeEngine([5])
    assert run_request(eng, {"input_ids": []})["finish_reason"] == "abort"
    r = run_request(eng, {"input_ids": [1], "sampling_params": {"max_new_tokens": 0}})
    assert r["finish_reason"] == "length" and r["output_ids"] == [] and not eng.calls


def test_greedy_seeded_sampling_and_finish_reasons():
    eng = FakeEngine([7, 8, 9, 2, 4])
    r = run_request(eng, {"input_ids": [1, 2], "sampling_params": {"max_new_tokens": 5, "top_k": 1}},
                    eos_id=2)
    assert eng.sampling_calls[-1] == (0.0, 1, 1.0, 0)          # greedy
    assert r["output_ids"] == [7, 8, 9, 2] and r["finish_reason"] == "stop" and r["seed"] is None
    r = run_request(eng, {"input_ids": [1], "sampling_params": {
        "max_new_tokens": 3, "temperature": 0.8, "top_p": 0.7, "sampling_seed": 11}})
    assert eng.sampling_calls[-1] == (0.8, 0, 0.7, 11)       # -1 (no top-k) -> 0
    assert r["finish_reason"] == "length" and r["output_ids"] == [7, 8, 9] and r["seed"] == 11
    r = run_request(eng, {"input_ids": [1], "sampling_params": {"max_new_tokens": 1, "top_p": 0.9}})
    assert r["seed"] is not None and eng.sampling_calls[-1][3] == r["seed"]   # fresh seed, reported
    assert eng.calls[-1] == ([1], 1, "loopspec", None)


def test_served_request_carries_its_generation_metrics():
    eng = FakeEngine([7, 8, 9, 10, 11])
    res = run_request(eng, {"input_ids": [1, 2], "sampling_params": {"max_new_tokens": 5, "top_k": 1}})
    m = res["metrics"]
    assert (m["decode_tokens"], m["decode_seconds"], m["decode_tok_s"]) == (4, 0.25, 16.0)
    assert (m["pipeline_cycles"], m["first_accept"], m["second_skip"]) == (10, 4, 0)
    aborted = run_request(eng, {"input_ids": [], "sampling_params": {}})
    assert aborted["metrics"] is None


def test_streamed_request_sends_every_unfinished_commit():
    eng = FakeEngine([7, 8, 9, 2, 11])
    sent = []
    req = {"input_ids": [1], "stream": True, "sampling_params": {"max_new_tokens": 5, "top_k": 1}}
    res = run_request(eng, req, eos_id=2, stream=sent.append)
    assert res["output_ids"] == [7, 8, 9, 2] and res["finish_reason"] == "stop"
    assert sent == [[7], [7, 8], [7, 8, 9]]        # the finishing commit is the return value
    sent.clear()
    run_request(eng, dict(req, stream=False), eos_id=2, stream=sent.append)
    assert sent == []                              # the request did not ask to stream


def test_divergent_engine_output_is_an_error():
    class Divergent(FakeEngine):
        def generate(self, ids, max_new, *, mode, stop_token=None, should_stop=None):
            out, st = super().generate(ids, max_new, mode=mode, stop_token=stop_token,
                                       should_stop=should_stop)
            return out[:-1] + [out[-1] + 1], st      # returns a token it never committed
    eng = Divergent([7, 8, 9])
    req = {"input_ids": [1], "stream": True, "sampling_params": {"max_new_tokens": 3, "top_k": 1}}
    with pytest.raises(RuntimeError, match="diverged"):
        run_request(eng, req, stream=lambda ids: None)
