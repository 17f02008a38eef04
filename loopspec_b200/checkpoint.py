"""Checkpoint tensors -> the engine's internal parameter names.

Restates the reference's checkpoint mapping for the two model families:

  Ouro   sglang_recurrent/modeling/ouro.py:19-34 (root prefixes and norm
         renames), :139-144 (map_ouro_weight), components.py:18-45 (split
         q/k/v and gate/up projections packed into qkv_proj / gate_up_proj)
  Raven  raven.py:24-58 (root prefixes, per-layout component renames),
         :193-197 (map_raven_weight)
  load   serving.py:142-182 (unmatched checkpoint tensors are reported, and
         raise only in strict mode)

The Ouro norm renames are one-to-one: `input_layernorm_2` -> the
post-attention norm, `post_attention_layernorm` -> the pre-feed-forward norm,
`post_attention_layernorm_2` -> the post-feed-forward norm. Each name is
mapped by exactly one rule, so a renamed norm is never renamed again.

`load_checkpoint` assembles the packed tensors (q rows, then k, then v; gate
rows, then up), checks every parameter the engine needs against
`weights.weight_shapes`, and returns {internal name: tensor} ready for
`Engine(...)`. The Ouro early-exit gate is accepted and dropped (the engine
does not run early exit).
"""

from __future__ import annotations

import glob
import logging
import os
from typing import Iterable

import torch

from .config import ModelConfig
from .weights import weight_shapes

log = logging.getLogger(__name__)

_OURO_PREFIX = {
    "model.embed_tokens.weight": "pre_executor.embed_tokens.weight",
    "model.norm.weight": "recurrent_executor.step_norm.weight",
    "model.early_exit_gate.": "recurrent_executor.early_exit_gate.",
    "model.layers.": "recurrent_executor.blocks.",
    "lm_head.weight": "post_executor.lm_head.weight",
}
_OURO_NORMS = {
    ".input_layernorm_2.": ".post_attention_layernorm.",
    ".post_attention_layernorm_2.": ".post_feedforward_layernorm.",
    ".post_attention_layernorm.": ".pre_feedforward_layernorm.",
}
_PACKED = {
    ".self_attn.q_proj.": (".self_attn.qkv_proj.", "q"),
    ".self_attn.k_proj.": (".self_attn.qkv_proj.", "k"),
    ".self_attn.v_proj.": (".self_attn.qkv_proj.", "v"),
    ".mlp.gate_proj.": (".mlp.gate_up_proj.", 0),
    ".mlp.up_proj.": (".mlp.gate_up_proj.", 1),
}
_RAVEN_PREFIX = {
    "transformer.prelude.": "pre_executor.blocks.",
    "transformer.core_block.": "recurrent_executor.blocks.",
    "transformer.coda.": "post_executor.blocks.",
    "transformer.wte.weight": "pre_executor.embed_tokens.weight",
    "transformer.adapter.weight": "recurrent_executor.adapter.weight",
    "transformer.adapter.bias": "recurrent_executor.adapter.bias",
    "transformer.ln_f.weight": "post_executor.final_norm.weight",
    "lm_head.weight": "post_executor.lm_head.weight",
}
_RAVEN_COMPONENTS = {
    ".attn.Wqkv.": ".self_attn.qkv_proj.",
    ".attn.proj.": ".self_attn.o_proj.",
    ".attn.q_norm.": ".self_attn.q_norm.",
    ".attn.k_norm.": ".self_attn.k_norm.",
    ".mlp.fc.": ".mlp.gate_up_proj.",
    ".mlp.proj.": ".mlp.down_proj.",
}
_RAVEN_NORMS = {
    "raven_pre": {".norm_1.": ".input_layernorm.", ".norm_2.": ".post_attention_layernorm."},
    "olmo_post": {".norm_1.": ".post_attention_layernorm.", ".norm_2.": ".post_feedforward_layernorm."},
}


def _prefix(name: str, rules: dict) -> str | None:
    for src, dst in rules.items():
        if name.startswith(src):
            return dst + name[len(src):]
    return None


def _substr_once(name: str, rules: dict) -> str:
    """Apply the first matching rule only (one-to-one renames)."""
    for src, dst in rules.items():
        if src in name:
            return name.replace(src, dst, 1)
    return name


def map_ouro_weight(name: str):
    """(internal name, shard) for an Ouro checkpoint name, or (None, None)."""
    target = _prefix(name, _OURO_PREFIX)
    if target is None:
        return None, None
    target = _substr_once(target, _OURO_NORMS)
    for src, (dst, shard) in _PACKED.items():
        if src in target:
            return target.replace(src, dst, 1), shard
    return target, None


def map_raven_weight(name: str, layout: str):
    """(internal name, None) for a Raven checkpoint name, or (None, None)."""
    target = _prefix(name, _RAVEN_PREFIX)
    if target is None:
        return None, None
    target = _substr_once(target, _RAVEN_COMPONENTS)
    return _substr_once(target, _RAVEN_NORMS[layout]), None


def load_checkpoint(tensors: Iterable[tuple[str, torch.Tensor]], cfg: ModelConfig, *,
                    device="cpu", dtype=torch.bfloat16, strict: bool = False) -> dict:
    """Map (checkpoint name, tensor) pairs to the engine's parameters.

    Raises ValueError for a missing parameter, a shape mismatch, or (strict)
    an unmatched checkpoint tensor; unmatched tensors are otherwise logged.
    """
    shapes = weight_shapes(cfg)
    out: dict[str, torch.Tensor] = {}
    shards: dict[str, dict] = {}
    unmatched: list[str] = []
    for name, t in tensors:
        if cfg.family == "ouro":
            target, shard = map_ouro_weight(name)
        else:
            target, shard = map_raven_weight(name, cfg.layout)
        if target is not None and target.startswith("recurrent_executor.early_exit_gate."):
            continue
        if target is None or target not in shapes:
            unmatched.append(name)
            continue
        if shard is None:
            out[target] = t
        else:
            shards.setdefault(target, {})[shard] = t
    for target, parts in shards.items():
        order = ("q", "k", "v") if "qkv_proj" in target else (0, 1)
        missing = [s for s in order if s not in parts]
        if missing:
            raise ValueError(f"{target}: checkpoint lacks shard(s) {missing}")
        out[target] = torch.cat([parts[s] for s in order], dim=0)
    if unmatched:
        msg = f"{len(unmatched)} checkpoint tensors were not matched; first entries: {unmatched[:8]}"
        if strict:
            raise ValueError(msg)
        log.warning(msg)
    missing = sorted(set(shapes) - set(out))
    if missing:
        raise ValueError(f"checkpoint lacks {len(missing)} parameters, e.g. {missing[:4]}")
    result = {}
    for name, shape in shapes.items():
        t = out[name]
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name}: checkpoint shape {tuple(t.shape)} != expected {tuple(shape)}")
        result[name] = t.to(device=device, dtype=dtype).contiguous()
    return result


def iter_safetensors(path: str):
    """(name, tensor) pairs of every *.safetensors file under `path` (or the file)."""
    from safetensors.torch import safe_open

    files = [path] if os.path.isfile(path) else sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no .safetensors files at {path}")
    for f in files:
        with safe_open(f, framework="pt") as h:
            for k in h.keys():
                yield k, h.get_tensor(k)
