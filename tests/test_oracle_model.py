"""Oracle model checks: layer math vs transformers, LoopSpec == AR self-consistency."""

import pytest
import torch

from loopspec_b200.config import get_config
from loopspec_b200.weights import init_random_weights
from oracle.executor import generate_ar_oracle, generate_loopspec_oracle
from oracle.model import OracleModel, Timeline, philox4x32, raven_initial_hidden
from oracle.pipeline import PipelineSchedule


def _tf_layer(layout, cfg, w, prefix):
    """Build the transformers layer equivalent to one oracle block."""
    if layout == "raven_pre":
        from transformers import LlamaConfig
        from transformers.models.llama.modeling_llama import LlamaDecoderLayer, LlamaRotaryEmbedding
        tc = LlamaConfig(hidden_size=cfg.hidden, num_attention_heads=cfg.n_heads,
                         num_key_value_heads=cfg.n_kv_heads, head_dim=cfg.head_dim,
                         intermediate_size=cfg.intermediate, rms_norm_eps=cfg.rms_eps,
                         rope_theta=cfg.rope_theta, attention_bias=False, mlp_bias=False)
        tc._attn_implementation = "eager"
        layer, rot = LlamaDecoderLayer(tc, 0), LlamaRotaryEmbedding(tc)
    else:
        from transformers import Olmo2Config
        from transformers.models.olmo2.modeling_olmo2 import Olmo2DecoderLayer, Olmo2RotaryEmbedding
        tc = Olmo2Config(hidden_size=cfg.hidden, num_attention_heads=cfg.n_heads,
                         num_key_value_heads=cfg.n_kv_heads, intermediate_size=cfg.intermediate,
                         rms_norm_eps=cfg.rms_eps, rope_theta=cfg.rope_theta, attention_bias=False)
        tc._attn_implementation = "eager"
        layer, rot = Olmo2DecoderLayer(tc, 0), Olmo2RotaryEmbedding(tc)
    nh, nkv, hd, I = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.intermediate
    qkv = w[prefix + "self_attn.qkv_proj.weight"]
    gu = w[prefix + "mlp.gate_up_proj.weight"]
    sd = {
        "self_attn.q_proj.weight": qkv[: nh * hd],
        "self_attn.k_proj.weight": qkv[nh * hd:(nh + nkv) * hd],
        "self_attn.v_proj.weight": qkv[(nh + nkv) * hd:],
        "self_attn.o_proj.weight": w[prefix + "self_attn.o_proj.weight"],
        "mlp.gate_proj.weight": gu[:I], "mlp.up_proj.weight": gu[I:],
        "mlp.down_proj.weight": w[prefix + "mlp.down_proj.weight"],
        "post_attention_layernorm.weight": w[prefix + "post_attention_layernorm.weight"],
    }
    if layout == "raven_pre":
        sd["input_layernorm.weight"] = w[prefix + "input_layernorm.weight"]
    else:
        sd["post_feedforward_layernorm.weight"] = w[prefix + "post_feedforward_layernorm.weight"]
        sd["self_attn.q_norm.weight"] = w[prefix + "self_attn.q_norm.weight"]
        sd["self_attn.k_norm.weight"] = w[prefix + "self_attn.k_norm.weight"]
    layer.load_state_dict(sd)
    return layer.eval(), rot


@pytest.mark.parametrize("name", ["tiny-raven-llama", "tiny-raven-olmo"])
def test_raven_layer_matches_transformers(name):
    cfg = get_config(name)
    w = init_random_weights(cfg, 3, dtype=torch.float32)
    # make norm weights non-trivial so norm placement is exercised
    g = torch.Generator().manual_seed(5)
    for k in list(w):
        if k.endswith("norm.weight"):
            w[k] = 1.0 + 0.1 * torch.randn(w[k].shape, generator=g)
    m = OracleModel(cfg.as_dict(), w)
    prefix = "recurrent_executor.blocks.0."
    layer, rot = _tf_layer(cfg.layout, cfg, w, prefix)
    L = 9
    x = torch.randn(1, L, cfg.hidden, generator=g)
    pos = torch.arange(L)[None]
    mask = torch.full((L, L), float("-inf")).triu(1)[None, None]
    with torch.no_grad():
        ref = layer(x, attention_mask=mask, position_ids=pos,
                    position_embeddings=rot(x, pos))
        ref = ref[0] if isinstance(ref, tuple) else ref
        tl = Timeline(1)
        got = torch.stack([m.layer(prefix, x[0, p], p, tl, 0) for p in range(L)])
    torch.testing.assert_close(got, ref[0], atol=2e-5, rtol=2e-5)


def test_philox_known_answer():
    # Random123 philox4x32-10 known-answer vectors (kat_vectors).
    import numpy as np
    ctr = np.array([[0, 0, 0, 0]], dtype=np.uint64)
    out = philox4x32(ctr, (0, 0))[0].tolist()
    assert out == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    ctr = np.array([[0xFFFFFFFF] * 4], dtype=np.uint64)
    out = philox4x32(ctr, (0xFFFFFFFF, 0xFFFFFFFF))[0].tolist()
    assert out == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]


def test_raven_hidden_init_is_position_keyed_and_truncated():
    a = raven_initial_hidden(7, 100, 512, 0.1, 2.0)
    b = raven_initial_hidden(7, 100, 512, 0.1, 2.0)
    c = raven_initial_hidden(7, 101, 512, 0.1, 2.0)
    assert torch.equal(a, b) and not torch.equal(a, c)
    assert a.abs().max() <= 0.3 * 2.0 + 1e-6
    assert abs(a.std().item() / 2.0 - 0.1) < 0.02


@pytest.mark.parametrize("name,K,X", [("tiny", 1, 2), ("tiny", 1, None), ("tiny", 2, None),
                                      ("tiny-raven-llama", 2, 2), ("tiny-raven-olmo", 1, 4)])
def test_oracle_loopspec_equals_ar(name, K, X):
    cfg = get_config(name)
    w = init_random_weights(cfg, 0, dtype=torch.float32)
    m = OracleModel(cfg.as_dict(), w)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab, (16,), generator=g).tolist()
    sch = PipelineSchedule(cfg.stages, K, X)
    ls, stats = generate_loopspec_oracle(m, sch, prompt, 12)
    ar = generate_ar_oracle(m, cfg.stages, prompt, 12)
    assert ls == ar
    assert stats["decode_tokens"] == 11
    assert stats["verified_proposals"] == stats["decode_tokens"]


def _ouro_tf_layer(cfg, w, prefix):
    """transformers' Gemma2DecoderLayer with Llama attention / MLP and plain
    RMSNorm modules swapped in, as the reference's OuroDecoderLayer subclasses
    SGLang's Gemma2DecoderLayer and replaces the same four parts
    (sglang_recurrent/modeling/ouro.py:37-82): Gemma2's residual flow, Llama's
    fused-QKV attention with neox RoPE and SiLU MLP, x * rsqrt(mean x^2 + eps) * w."""
    from transformers import Gemma2Config, LlamaConfig
    from transformers.models.gemma2.modeling_gemma2 import Gemma2DecoderLayer
    from transformers.models.llama.modeling_llama import (LlamaAttention, LlamaMLP, LlamaRMSNorm,
                                                          LlamaRotaryEmbedding)
    lc = LlamaConfig(hidden_size=cfg.hidden, num_attention_heads=cfg.n_heads,
                     num_key_value_heads=cfg.n_kv_heads, head_dim=cfg.head_dim,
                     intermediate_size=cfg.intermediate, rms_norm_eps=cfg.rms_eps,
                     rope_theta=cfg.rope_theta, attention_bias=False, mlp_bias=False)
    lc._attn_implementation = "eager"
    gc = Gemma2Config(hidden_size=cfg.hidden, num_attention_heads=cfg.n_heads,
                      num_key_value_heads=cfg.n_kv_heads, head_dim=cfg.head_dim,
                      intermediate_size=cfg.intermediate, rms_norm_eps=cfg.rms_eps)
    gc._attn_implementation = "eager"
    layer = Gemma2DecoderLayer(gc, 0)
    layer.self_attn = LlamaAttention(lc, 0)
    layer.mlp = LlamaMLP(lc)
    for name in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                 "post_feedforward_layernorm"):
        setattr(layer, name, LlamaRMSNorm(cfg.hidden, eps=cfg.rms_eps))
    nh, nkv, hd, I = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.intermediate
    qkv = w[prefix + "self_attn.qkv_proj.weight"]
    gu = w[prefix + "mlp.gate_up_proj.weight"]
    sd = {
        "self_attn.q_proj.weight": qkv[: nh * hd],
        "self_attn.k_proj.weight": qkv[nh * hd:(nh + nkv) * hd],
        "self_attn.v_proj.weight": qkv[(nh + nkv) * hd:],
        "self_attn.o_proj.weight": w[prefix + "self_attn.o_proj.weight"],
        "mlp.gate_proj.weight": gu[:I], "mlp.up_proj.weight": gu[I:],
        "mlp.down_proj.weight": w[prefix + "mlp.down_proj.weight"],
    }
    for name in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                 "post_feedforward_layernorm"):
        sd[name + ".weight"] = w[prefix + name + ".weight"]
    layer.load_state_dict(sd)
    return layer.eval(), LlamaRotaryEmbedding(lc)


def test_ouro_layer_matches_the_gemma2_residual_flow():
    cfg = get_config("tiny")
    w = init_random_weights(cfg, 3, dtype=torch.float32)
    g = torch.Generator().manual_seed(6)
    for k in list(w):
        if k.endswith("norm.weight"):
            w[k] = 1.0 + 0.1 * torch.randn(w[k].shape, generator=g)
    m = OracleModel(cfg.as_dict(), w)
    prefix = "recurrent_executor.blocks.1."
    layer, rot = _ouro_tf_layer(cfg, w, prefix)
    L = 9
    x = torch.randn(1, L, cfg.hidden, generator=g)
    pos = torch.arange(L)[None]
    mask = torch.full((L, L), float("-inf")).triu(1)[None, None]
    with torch.no_grad():
        ref = layer(x, attention_mask=mask, position_ids=pos, position_embeddings=rot(x, pos))
        ref = ref[0] if isinstance(ref, tuple) else ref
        tl = Timeline(1)
        got = torch.stack([m.layer(prefix, x[0, p], p, tl, 0) for p in range(L)])
    torch.testing.assert_close(got, ref[0], atol=2e-5, rtol=2e-5)
