"""Request semantics of the reference's LoopSpec scheduler, without the server.

Restates sglang_recurrent/server/loopspec_scheduler.py for one already
tokenized request:
  _unsupported_options (:49-148)  features LoopSpec does not implement abort
                                  the request, naming them, before any model
                                  work;
  _run_request (:288-375)         an empty prompt aborts; max_new_tokens == 0
                                  finishes with length 0 and no model work;
                                  top_k == 1 (SGLang's greedy normalisation)
                                  selects greedy decisions, otherwise
                                  temperature / top_k / top_p sampling keyed by
                                  the request's sampling_seed; generation ends
                                  at the EOS id or at max_new_tokens; a served
                                  request yields its generation_metrics record
                                  (:364-375, server/metrics.py).
The HTTP server, tokenizer and detokenizer processes, streaming transport and
stop strings stay out of scope (they need SGLang's request objects). Field
names follow SGLang's tokenized request and its sampling_params.
"""

from __future__ import annotations

import secrets
from typing import Any, Sequence

from .executor import apply_sampling
from .metrics import request_metrics

_ROUTING = ("bootstrap_host", "bootstrap_port", "bootstrap_room", "bootstrap_pair_key",
            "decode_tp_size", "routed_dp_rank", "disagg_prefill_dp_rank")


def unsupported_options(request: dict) -> list[str]:
    """Names of requested features LoopSpec does not implement (empty list: none),
    in the reference's order."""
    r, p = request, request.get("sampling_params") or {}
    checks = [
        (r.get("mm_inputs"), "multimodal input"),
        (any(r.get(k) for k in ("need_wait_for_mm_inputs", "num_items_assigned",
                                "mm_data_mooncake", "encoder_urls")), "multimodal IPC state"),
        (r.get("input_embeds") is not None, "input_embeds"),
        (r.get("token_type_ids") is not None, "token_type_ids"),
        (r.get("session_params") is not None, "sessions"),
        (r.get("lora_id") is not None, "LoRA"),
        (any(r.get(k) is not None for k in _ROUTING), "distributed request routing"),
        (r.get("return_logprob"), "return_logprob"),
        (r.get("return_hidden_states"), "return_hidden_states"),
        (r.get("return_routed_experts"), "return_routed_experts"),
        (r.get("return_indexer_topk"), "return_indexer_topk"),
        (r.get("return_entropy"), "return_entropy"),
        (r.get("return_bytes"), "return_bytes"),
        (r.get("custom_logit_processor") is not None, "custom_logit_processor"),
        (r.get("positional_embed_overrides") is not None, "positional_embed_overrides"),
        (r.get("require_reasoning"), "hybrid reasoning"),
        (r.get("multi_item_delimiter_indices") is not None, "multi-item scoring"),
        (any(p.get(k) for k in ("json_schema", "regex", "ebnf", "structural_tag")),
         "constrained decoding"),
        (p.get("logit_bias"), "logit_bias"),
        (p.get("custom_params"), "custom sampling parameters"),
        (p.get("min_p", 0) != 0, "min_p"),
        (p.get("min_new_tokens", 0) != 0, "min_new_tokens"),
        ("max_new_tokens" in p and p["max_new_tokens"] is None, "unbounded max_new_tokens"),
        (r.get("stream") and p.get("stream_interval") not in (None, 1), "stream_interval other than 1"),
        (p.get("frequency_penalty", 0) != 0 or p.get("presence_penalty", 0) != 0
         or p.get("repetition_penalty", 1) != 1, "sampling penalties"),
    ]
    return [label for hit, label in checks if hit]


def run_request(engine: Any, request: dict, eos_id: int | None = None, stream=None) -> dict:
    """Serve one tokenized request on `engine` (a loopspec_b200.engine.Engine).

    request = {"input_ids": [...], "sampling_params": {...}, ...}. Returns
    {"output_ids", "finish_reason" ("abort" | "length" | "stop"), "message",
    "seed" (the sampling stream used, None for greedy), "stats", "metrics"
    (the generation_metrics fields; None when no model work ran)}. A sampled
    request without sampling_seed draws a fresh seed, as the reference draws
    from the device's default generator. When the request asks to stream and
    `stream` is given, stream(ids) receives the whole committed output after
    every commit that does not finish the request (interval 1,
    loopspec_scheduler.py:331-346); the finished output is the return value.
    """
    def done(reason, message="", ids=(), seed=None, stats=None):
        return {"output_ids": list(ids), "finish_reason": reason, "message": message,
                "seed": seed, "stats": stats or {},
                "metrics": request_metrics(list(ids), stats) if stats else None}

    unsupported = unsupported_options(request)
    if unsupported:
        return done("abort", "LoopSpec does not support: " + ", ".join(unsupported))
    ids: Sequence[int] = request.get("input_ids") or []
    if not ids:
        return done("abort", "LoopSpec requires a nonempty prompt")
    p = request.get("sampling_params") or {}
    max_new = int(p.get("max_new_tokens", 128))
    if max_new == 0:
        return done("length")
    seed = None
    if p.get("top_k", -1) == 1:
        apply_sampling(engine, None)
    else:
        seed = p.get("sampling_seed")
        seed = secrets.randbits(63) if seed is None else int(seed)
        # SGLang writes "no top-k" as -1, the engine as 0
        apply_sampling(engine, {"temperature": p.get("temperature", 1.0),
                                "top_k": max(0, int(p.get("top_k", -1))),
                                "top_p": p.get("top_p", 1.0)}, seed=seed)
    should_stop = None
    seen: list = []
    if stream is not None and request.get("stream"):
        def should_stop(committed):
            seen[:] = committed
            finished = len(committed) >= max_new or (eos_id is not None and committed[-1] == eos_id)
            if not finished:
                stream(list(committed))
            return False
    out, stats = engine.generate(list(ids), max_new, mode="loopspec", stop_token=eos_id,
                                 should_stop=should_stop)
    # the callback and the executor must agree on the whole committed sequence
    # (loopspec_scheduler.py:356-358)
    if should_stop is not None and list(seen) != list(out):
        raise RuntimeError("LoopSpec request state diverged from pipeline output")
    reason = "stop" if eos_id is not None and out and out[-1] == eos_id else "length"
    return done(reason, ids=out, seed=seed, stats=stats)
