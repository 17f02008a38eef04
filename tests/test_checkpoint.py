"""Checkpoint name mapping (loopspec_b200.checkpoint) against the reference's
rules (ouro.py:19-34,139-144; raven.py:24-58,193-197; components.py:18-45).

Synthetic checkpoints are built from seeded internal weights by the inverse
renames; every norm gets distinct random values so a swapped rename shows.
"""

import pytest
import torch

from loopspec_b200.checkpoint import (iter_safetensors, load_checkpoint, map_ouro_weight,
                                      map_raven_weight)
from loopspec_b200.config import get_config
from loopspec_b200.weights import weight_shapes


def internal_weights(cfg, seed=0):
    g = torch.Generator().manual_seed(seed)
    return {n: torch.randn(s, generator=g) for n, s in sorted(weight_shapes(cfg).items())}


def ouro_checkpoint(cfg, w):
    norms = {"input_layernorm": "input_layernorm", "post_attention_layernorm": "input_layernorm_2",
             "pre_feedforward_layernorm": "post_attention_layernorm",
             "post_feedforward_layernorm": "post_attention_layernorm_2"}
    qd, kd = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    ck = {"model.embed_tokens.weight": w["pre_executor.embed_tokens.weight"],
          "model.norm.weight": w["recurrent_executor.step_norm.weight"],
          "lm_head.weight": w["post_executor.lm_head.weight"],
          "model.early_exit_gate.weight": torch.zeros(1, cfg.hidden),
          "model.early_exit_gate.bias": torch.zeros(1)}
    for i in range(cfg.n_core_layers):
        p, q = f"recurrent_executor.blocks.{i}.", f"model.layers.{i}."
        qkv = w[p + "self_attn.qkv_proj.weight"]
        ck[q + "self_attn.q_proj.weight"] = qkv[:qd]
        ck[q + "self_attn.k_proj.weight"] = qkv[qd:qd + kd]
        ck[q + "self_attn.v_proj.weight"] = qkv[qd + kd:]
        gu = w[p + "mlp.gate_up_proj.weight"]
        ck[q + "mlp.gate_proj.weight"] = gu[:cfg.intermediate]
        ck[q + "mlp.up_proj.weight"] = gu[cfg.intermediate:]
        ck[q + "self_attn.o_proj.weight"] = w[p + "self_attn.o_proj.weight"]
        ck[q + "mlp.down_proj.weight"] = w[p + "mlp.down_proj.weight"]
        for internal, hf in norms.items():
            ck[q + hf + ".weight"] = w[p + internal + ".weight"]
    return ck


def raven_checkpoint(cfg, w):
    prefix = {"pre_executor.blocks.": "transformer.prelude.",
              "recurrent_executor.blocks.": "transformer.core_block.",
              "post_executor.blocks.": "transformer.coda.",
              "pre_executor.embed_tokens.weight": "transformer.wte.weight",
              "recurrent_executor.adapter.weight": "transformer.adapter.weight",
              "recurrent_executor.adapter.bias": "transformer.adapter.bias",
              "post_executor.final_norm.weight": "transformer.ln_f.weight",
              "post_executor.lm_head.weight": "lm_head.weight"}
    comp = {".self_attn.qkv_proj.": ".attn.Wqkv.", ".self_attn.o_proj.": ".attn.proj.",
            ".self_attn.q_norm.": ".attn.q_norm.", ".self_attn.k_norm.": ".attn.k_norm.",
            ".mlp.gate_up_proj.": ".mlp.fc.", ".mlp.down_proj.": ".mlp.proj."}
    norms = ({".input_layernorm.": ".norm_1.", ".post_attention_layernorm.": ".norm_2."}
             if cfg.layout == "raven_pre" else
             {".post_attention_layernorm.": ".norm_1.", ".post_feedforward_layernorm.": ".norm_2."})
    ck = {}
    for name, t in w.items():
        out = name
        for a, b in prefix.items():
            if out.startswith(a):
                out = b + out[len(a):]
                break
        for a, b in {**comp, **norms}.items():
            if a in out:
                out = out.replace(a, b, 1)
                break
        ck[out] = t
    return ck


def test_ouro_rules_match_the_reference_table():
    assert map_ouro_weight("model.layers.3.self_attn.k_proj.weight") == \
        ("recurrent_executor.blocks.3.self_attn.qkv_proj.weight", "k")
    assert map_ouro_weight("model.layers.0.mlp.up_proj.weight") == \
        ("recurrent_executor.blocks.0.mlp.gate_up_proj.weight", 1)
    assert map_ouro_weight("model.layers.1.input_layernorm_2.weight")[0] == \
        "recurrent_executor.blocks.1.post_attention_layernorm.weight"
    assert map_ouro_weight("model.layers.1.post_attention_layernorm.weight")[0] == \
        "recurrent_executor.blocks.1.pre_feedforward_layernorm.weight"
    assert map_ouro_weight("model.layers.1.post_attention_layernorm_2.weight")[0] == \
        "recurrent_executor.blocks.1.post_feedforward_layernorm.weight"
    assert map_ouro_weight("model.layers.1.input_layernorm.weight")[0] == \
        "recurrent_executor.blocks.1.input_layernorm.weight"
    assert map_ouro_weight("model.rotary_emb.inv_freq") == (None, None)


def test_raven_rules_match_the_reference_table():
    assert map_raven_weight("transformer.core_block.2.attn.Wqkv.weight", "raven_pre")[0] == \
        "recurrent_executor.blocks.2.self_attn.qkv_proj.weight"
    assert map_raven_weight("transformer.coda.0.norm_2.weight", "raven_pre")[0] == \
        "post_executor.blocks.0.post_attention_layernorm.weight"
    assert map_raven_weight("transformer.coda.0.norm_2.weight", "olmo_post")[0] == \
        "post_executor.blocks.0.post_feedforward_layernorm.weight"
    assert map_raven_weight("transformer.ln_f.weight", "olmo_post")[0] == "post_executor.final_norm.weight"
    assert map_raven_weight("transformer.freqs_cis", "raven_pre") == (None, None)


@pytest.mark.parametrize("name", ["tiny", "tiny-raven-llama", "tiny-raven-olmo"])
def test_checkpoint_round_trip(name):
    cfg = get_config(name)
    w = internal_weights(cfg)
    ck = ouro_checkpoint(cfg, w) if cfg.family == "ouro" else raven_checkpoint(cfg, w)
    got = load_checkpoint(ck.items(), cfg, dtype=torch.float32, strict=True)
    assert set(got) == set(w)
    for k in w:
        assert torch.equal(got[k], w[k]), k


def test_unmatched_missing_and_bad_shapes_are_reported(caplog):
    cfg = get_config("tiny")
    w = internal_weights(cfg)
    ck = ouro_checkpoint(cfg, w)
    ck["model.rotary_emb.inv_freq"] = torch.zeros(32)
    load_checkpoint(ck.items(), cfg, dtype=torch.float32)          # logged, not raised
    assert "not matched" in caplog.text
    with pytest.raises(ValueError, match="not matched"):
        load_checkpoint(ck.items(), cfg, dtype=torch.float32, strict=True)
    del ck["model.rotary_emb.inv_freq"]
    bad = dict(ck)
    del bad["model.layers.0.self_attn.v_proj.weight"]
    with pytest.raises(ValueError, match="shard"):
        load_checkpoint(bad.items(), cfg, dtype=torch.float32)
    bad = dict(ck)
    del bad["model.norm.weight"]
    with pytest.raises(ValueError, match="lacks"):
        load_checkpoint(bad.items(), cfg, dtype=torch.float32)
    bad = dict(ck)
    bad["model.layers.1.mlp.down_proj.weight"] = torch.zeros(3, 3)
    with pytest.raises(ValueError, match="shape"):
        load_checkpoint(bad.items(), cfg, dtype=torch.float32)


def test_safetensors_files_load(tmp_path):
    from safetensors.torch import save_file
    cfg = get_config("tiny")
    w = internal_weights(cfg)
    ck = {k: v.contiguous() for k, v in ouro_checkpoint(cfg, w).items()}
    names = sorted(ck)
    save_file({k: ck[k] for k in names[: len(names) // 2]}, str(tmp_path / "a.safetensors"))
    save_file({k: ck[k] for k in names[len(names) // 2:]}, str(tmp_path / "b.safetensors"))
    got = load_checkpoint(iter_safetensors(str(tmp_path)), cfg, dtype=torch.bfloat16)
    for k in w:
        assert torch.equal(got[k], w[k].to(torch.bfloat16)), k


def test_config_from_hf_reads_both_families():
    import math
    from loopspec_b200.config import config_from_hf
    ouro = config_from_hf({"model_type": "ouro", "hidden_size": 2048, "num_attention_heads": 16,
                           "num_key_value_heads": 16, "intermediate_size": 5632, "vocab_size": 49152,
                           "num_hidden_layers": 24, "total_ut_steps": 4, "rope_theta": 10000.0,
                           "rms_norm_eps": 1e-6, "tie_word_embeddings": False})
    ref = get_config("ouro-1.4b")
    for f in ("hidden", "n_heads", "n_kv_heads", "head_dim", "intermediate", "vocab",
              "n_core_layers", "stages", "family", "layout"):
        assert getattr(ouro, f) == getattr(ref, f), f
    rav = config_from_hf({"model_type": "huginn_raven", "n_embd": 5280, "n_heads": 55,
                          "num_key_value_heads": 55, "intermediate_size": 17920, "vocab_size": 65536,
                          "n_layers_in_prelude": 2, "n_layers_in_recurrent_block": 4,
                          "n_layers_in_coda": 2, "mean_recurrence": 32, "rope_base": 50000,
                          "norm_eps": 1e-6, "bias": False, "tie_embeddings": True})
    assert rav.layout == "raven_pre" and rav.head_dim == 96 and rav.stages == 32
    assert rav.embed_scale == pytest.approx(math.sqrt(5280))
    assert rav.init_std == pytest.approx(math.sqrt(2 / (5 * 5280)))
    olmo = config_from_hf({"model_type": "huginn_raven", "n_embd": 2048, "n_heads": 16,
                           "head_dim": 128, "intermediate_size": 8192, "vocab_size": 100352,
                           "n_layers_in_prelude": 2, "n_layers_in_recurrent_block": 4,
                           "n_layers_in_coda": 2, "mean_recurrence": 32,
                           "rope_parameters": {"rope_theta": 500000.0}, "norm_eps": 1e-6})
    assert olmo.layout == "olmo_post" and olmo.qk_norm and olmo.rope_theta == 500000.0
    with pytest.raises(ValueError, match="test_time_noise"):
        config_from_hf({"model_type": "huginn_raven", "test_time_noise": 0.1, "n_embd": 8, "n_heads": 2})
    with pytest.raises(ValueError, match="unsupported"):
        config_from_hf({"model_type": "llama"})
