"""Byte accounting of the decode roofline (CPU)."""

from loopspec_b200 import roofline
from loopspec_b200.config import get_config


def ar_stats(cfg, prompt_len, n):
    """Counters an autoregressive decode of n tokens produces: one pre, S
    core and one post call per token; the core lane of token i attends to
    prompt_len + i positions at each depth."""
    S = cfg.stages
    return {"core_calls": S * n, "pre_calls": n if cfg.n_pre_layers else 0, "post_calls": n,
            "recurrent_rows": S * n,
            "core_kv_positions": S * sum(prompt_len + i for i in range(1, n + 1))}


def test_ar_decode_moves_exactly_the_useful_bytes():
    for name in ("ouro-1.4b", "raven-olmo", "tiny"):
        cfg = get_config(name)
        st = ar_stats(cfg, 512, 1023)
        assert roofline.decode_bytes(cfg, st) == roofline.useful_bytes(cfg, 1023, 512)


def test_ouro_1p4b_ar_bytes_per_token_match_the_per_token_formula():
    cfg = get_config("ouro-1.4b")
    w_core, w_pre, w_post, w_lm = roofline.weight_bytes(cfg)
    assert abs(w_core - 2.466e9) < 5e6 and abs(w_lm - 0.201e9) < 1e6 and w_pre == w_post == 0
    per_tok = roofline.useful_bytes(cfg, 1, 1023)     # one token at context 1024
    # 4 core iterations + lm_head + K/V of 1024 positions at 4 depths (+ the new row)
    assert per_tok == 4 * w_core + w_lm + 4 * 196608 * 1025
    assert 10.8e9 < per_tok < 11.0e9


def test_counters_sum_over_requests():
    cfg = get_config("ouro-1.4b")
    a, b = ar_stats(cfg, 100, 10), ar_stats(cfg, 300, 20)
    both = {k: a[k] + b[k] for k in a}
    assert roofline.decode_bytes(cfg, both) == roofline.decode_bytes(cfg, a) + roofline.decode_bytes(cfg, b)


def test_batched_useful_bytes_stream_weights_once_per_step():
    cfg = get_config("ouro-1.4b")
    one = roofline.useful_bytes(cfg, 100, 500)
    assert roofline.useful_bytes_batch(cfg, [100], [500]) == one
    two = roofline.useful_bytes_batch(cfg, [100, 100], [500, 500])
    kv = one - 100 * sum(roofline.weight_bytes(cfg)[i] * (cfg.stages if i == 0 else 1) for i in range(4))
    assert two == one + kv                      # the second request adds only its K/V
