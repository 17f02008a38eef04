"""Seeded random weights with the reference's internal parameter names.

Names are those of RecurrentServingModel after checkpoint mapping
(sglang_recurrent/modeling/ouro.py:19-34, raven.py:221-255,
components.py:18-45): packed `qkv_proj` (q rows, then k, then v) and packed
`gate_up_proj` (gate rows, then up). Linear and embedding weights are
N(0, 0.02); norm weights are 1; the adapter bias (if any) is 0. Tensors are
drawn in sorted-name order from one torch.Generator seeded with `seed` on
`device`, in float32, then cast to `dtype`.
"""

from __future__ import annotations

import torch

from .config import ModelConfig


def weight_shapes(cfg: ModelConfig) -> dict[str, tuple[int, ...]]:
    H, I, V = cfg.hidden, cfg.intermediate, cfg.vocab
    shapes: dict[str, tuple[int, ...]] = {
        "pre_executor.embed_tokens.weight": (V, H),
    }
    if not cfg.tie_embeddings:
        shapes["post_executor.lm_head.weight"] = (V, H)

    def block(prefix):
        shapes[prefix + "self_attn.qkv_proj.weight"] = (cfg.qkv_dim, H)
        shapes[prefix + "self_attn.o_proj.weight"] = (H, cfg.n_heads * cfg.head_dim)
        shapes[prefix + "mlp.gate_up_proj.weight"] = (2 * I, H)
        shapes[prefix + "mlp.down_proj.weight"] = (H, I)
        if cfg.layout == "ouro":
            norms = ("input_layernorm", "post_attention_layernorm",
                     "pre_feedforward_layernorm", "post_feedforward_layernorm")
        elif cfg.layout == "raven_pre":
            norms = ("input_layernorm", "post_attention_layernorm")
        else:
            norms = ("post_attention_layernorm", "post_feedforward_layernorm")
        for n in norms:
            shapes[prefix + n + ".weight"] = (H,)
        if cfg.qk_norm:
            shapes[prefix + "self_attn.q_norm.weight"] = (cfg.n_heads * cfg.head_dim,)
            shapes[prefix + "self_attn.k_norm.weight"] = (cfg.n_kv_heads * cfg.head_dim,)

    for i in range(cfg.n_pre_layers):
        block(f"pre_executor.blocks.{i}.")
    for i in range(cfg.n_core_layers):
        block(f"recurrent_executor.blocks.{i}.")
    for i in range(cfg.n_post_layers):
        block(f"post_executor.blocks.{i}.")
    if cfg.family == "ouro":
        shapes["recurrent_executor.step_norm.weight"] = (H,)
    else:
        shapes["recurrent_executor.adapter.weight"] = (H, 2 * H)
        if cfg.adapter_bias:
            shapes["recurrent_executor.adapter.bias"] = (H,)
        shapes["post_executor.final_norm.weight"] = (H,)
    return shapes


def is_norm(name: str) -> bool:
    return "norm" in name.rsplit(".", 2)[-2] or name.endswith("step_norm.weight")


def init_random_weights(cfg: ModelConfig, seed: int = 0, device="cpu",
                        dtype=torch.bfloat16, std: float = 0.02):
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out = {}
    for name, shape in sorted(weight_shapes(cfg).items()):
        if is_norm(name):
            t = torch.ones(shape, device=device, dtype=torch.float32)
        elif name.endswith(".bias"):
            t = torch.zeros(shape, device=device, dtype=torch.float32)
        else:
            t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
            t.mul_(std)
        out[name] = t.to(dtype)
    return out
