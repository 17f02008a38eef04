"""HBM bytes of a decode loop, for the bytes-moved roofline.

The decode step streams weights and reads KV rows; its activations are a few
KB per lane. Two byte counts are reported against a decode's device time:

* ``decode_bytes``: what the loop actually moved, from the engine's work
  counters (``ls_stats``): every core call streams one iteration of core
  weights, every pre call with prelude layers streams the prelude, every post
  call streams the coda and the lm_head, and every core lane reads its
  timeline's K/V rows in every core layer and writes one row per layer.
  Rejected lanes count too: this is the work the GPU did.
* ``useful_bytes``: what autoregressive decoding of the committed tokens
  would move (S core iterations, prelude, coda and lm_head per token, and the
  K/V of S core depths at each token's context). Its fraction is the decode's
  speed expressed as the AR roofline.

Both follow the per-cycle formula K*W_core + [pre]*W_pre + [post]*(W_post +
W_lm) + sum over lanes and core layers of KV(L) (algorithmic bytes of
sglang_recurrent's decode cycle, executor.py:293-367 / serving.py:185-239).
"""

from __future__ import annotations


def weight_bytes(cfg):
    """(core iteration, prelude, coda, lm_head) weight bytes, bf16."""
    layer = cfg.layer_weight_bytes()
    return (cfg.core_weight_bytes(), cfg.n_pre_layers * layer, cfg.n_post_layers * layer,
            cfg.vocab * cfg.hidden * 2)


def decode_bytes(cfg, stats):
    """Bytes the decode loop moved, from its work counters (summable over requests)."""
    w_core, w_pre, w_post, w_lm = weight_bytes(cfg)
    kv_row = cfg.n_core_layers * cfg.kv_bytes_per_token_layer()
    core_lanes = stats["recurrent_rows"]
    return (stats["core_calls"] * w_core + stats["pre_calls"] * w_pre
            + stats["post_calls"] * (w_post + w_lm)
            + stats["core_kv_positions"] * kv_row + core_lanes * kv_row)


def useful_bytes(cfg, decode_tokens, prompt_len):
    """Bytes autoregressive decoding of `decode_tokens` tokens after a
    `prompt_len`-token prompt moves: token i (1-based) attends to prompt_len + i
    positions at each of the S core depths."""
    w_core, w_pre, w_post, w_lm = weight_bytes(cfg)
    S = cfg.stages
    kv_row = cfg.n_core_layers * cfg.kv_bytes_per_token_layer()
    n = decode_tokens
    positions = n * prompt_len + n * (n + 1) // 2
    return n * (S * w_core + w_pre + w_post + w_lm) + S * kv_row * (positions + n)


def useful_bytes_batch(cfg, decode_tokens, prompt_lens):
    """Bytes batched autoregressive decoding of several requests moves: each
    step streams the weights once for every request still running (so
    max(decode_tokens) weight passes), and each request reads its own K/V."""
    if not decode_tokens:
        return 0
    w_core, w_pre, w_post, w_lm = weight_bytes(cfg)
    S = cfg.stages
    kv_row = cfg.n_core_layers * cfg.kv_bytes_per_token_layer()
    steps = max(decode_tokens)
    kv = 0
    for n, P in zip(decode_tokens, prompt_lens):
        kv += S * kv_row * (n * P + n * (n + 1) // 2 + n)
    return steps * (S * w_core + w_pre + w_post + w_lm) + kv
