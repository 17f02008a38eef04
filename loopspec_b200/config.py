"""Model and schedule configurations for the looped decoders this engine serves.

Field meanings follow the reference's HF configs as read by
sglang_recurrent/modeling/{ouro,raven,contracts}.py: Ouro = embedding-only
pre, `n_core_layers` sandwich-norm layers + step_norm looped `stages` times,
lm_head-only post; Raven = prelude / adapter + core / coda + final norm, with
block layout "raven_pre" (Llama pre-norm) or "olmo_post" (OLMo2 post-norm +
QK-norm) chosen by head_dim == 128 (contracts.py:196).
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, replace


@dataclass(frozen=True)
class ModelConfig:
    name: str
    family: str                 # "ouro" | "raven"
    layout: str                 # "ouro" | "raven_pre" | "olmo_post"
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    n_pre_layers: int
    n_core_layers: int
    n_post_layers: int
    stages: int                 # S: total_ut_steps (Ouro) / mean_recurrence (Raven)
    rope_theta: float = 10000.0
    rms_eps: float = 1e-6
    embed_scale: float = 1.0
    init_std: float = 0.0       # Raven recurrent hidden init std; 0 for Ouro
    init_seed: int = 0          # Raven position-keyed hidden init seed
    qk_norm: bool = False
    adapter_bias: bool = False
    tie_embeddings: bool = False

    def as_dict(self):
        return asdict(self)

    @property
    def qkv_dim(self):
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    def core_weight_bytes(self, elem=2):
        """Bytes of one core iteration's weights (adapter included)."""
        H, I = self.hidden, self.intermediate
        per_layer = H * self.qkv_dim + self.n_heads * self.head_dim * H + 2 * I * H + I * H
        adapter = 2 * H * H if self.family == "raven" else 0
        return (self.n_core_layers * per_layer + adapter) * elem

    def layer_weight_bytes(self, elem=2):
        H, I = self.hidden, self.intermediate
        return (H * self.qkv_dim + self.n_heads * self.head_dim * H + 3 * I * H) * elem

    def kv_bytes_per_token_layer(self, elem=2):
        return 2 * self.n_kv_heads * self.head_dim * elem


def _raven(name, layout, heads, kv, hd, inter, vocab, **kw):
    H = 2048
    std = math.sqrt(2 / (5 * H))
    return ModelConfig(
        name=name, family="raven", layout=layout, hidden=H, n_heads=heads,
        n_kv_heads=kv, head_dim=hd, intermediate=inter, vocab=vocab,
        n_pre_layers=2, n_core_layers=4, n_post_layers=2, stages=32,
        rope_theta=50000.0, embed_scale=math.sqrt(H), init_std=std, **kw)


PRESETS = {
    # BASELINE.json configs[0]
    "tiny": ModelConfig(
        name="tiny-ouro", family="ouro", layout="ouro", hidden=256, n_heads=4,
        n_kv_heads=4, head_dim=64, intermediate=704, vocab=4096,
        n_pre_layers=0, n_core_layers=2, n_post_layers=0, stages=4),
    # configs[1]
    "ouro-1.4b": ModelConfig(
        name="ouro-1.4b", family="ouro", layout="ouro", hidden=2048, n_heads=16,
        n_kv_heads=16, head_dim=128, intermediate=5632, vocab=49152,
        n_pre_layers=0, n_core_layers=24, n_post_layers=0, stages=4),
    # configs[2]
    "ouro-2.6b": ModelConfig(
        name="ouro-2.6b", family="ouro", layout="ouro", hidden=2048, n_heads=16,
        n_kv_heads=16, head_dim=128, intermediate=5632, vocab=49152,
        n_pre_layers=0, n_core_layers=48, n_post_layers=0, stages=4),
    # configs[3]
    "raven-llama": _raven("raven-llama", "raven_pre", 32, 8, 64, 8192, 128256),
    # configs[4]
    "raven-olmo": _raven("raven-olmo", "olmo_post", 16, 16, 128, 8192, 100352, qk_norm=True),
    # small Raven shapes for CPU-oracle parity tests
    "tiny-raven-llama": ModelConfig(
        name="tiny-raven-llama", family="raven", layout="raven_pre", hidden=256,
        n_heads=4, n_kv_heads=1, head_dim=64, intermediate=512, vocab=4096,
        n_pre_layers=1, n_core_layers=2, n_post_layers=1, stages=8,
        rope_theta=50000.0, embed_scale=16.0, init_std=math.sqrt(2 / (5 * 256))),
    "tiny-raven-olmo": ModelConfig(
        name="tiny-raven-olmo", family="raven", layout="olmo_post", hidden=256,
        n_heads=2, n_kv_heads=2, head_dim=128, intermediate=512, vocab=4096,
        n_pre_layers=1, n_core_layers=2, n_post_layers=1, stages=8,
        rope_theta=50000.0, embed_scale=16.0, init_std=math.sqrt(2 / (5 * 256)),
        qk_norm=True),
}


def config_from_hf(hf: dict, name: str | None = None) -> ModelConfig:
    """ModelConfig from a checkpoint's HF config (config.json as a dict).

    Follows the reference's reading of the two model types:
    contracts.py:28-53 (family by model_type; Raven layout olmo_post iff
    head_dim == 128), contracts.py:56-65 (S = total_ut_steps / mean_recurrence),
    raven.py:87-187 (norm_eps, bias, prelude/core/coda layer counts,
    init_values embed_scale and std, RoPE base from rope_parameters /
    rope_theta / rope_base; nonzero test_time_noise is rejected) and
    integrations/huggingface.py:112-179 (Raven defaults: head_dim = n_embd /
    n_heads, std = sqrt(2 / (5 n_embd)), embed_scale = sqrt(n_embd)).
    """
    mt = hf.get("model_type")
    rope = (hf.get("rope_parameters") or {}).get("rope_theta")
    if mt == "ouro":
        H, heads = hf["hidden_size"], hf["num_attention_heads"]
        return ModelConfig(
            name=name or "ouro", family="ouro", layout="ouro", hidden=H, n_heads=heads,
            n_kv_heads=hf.get("num_key_value_heads") or heads,
            head_dim=hf.get("head_dim") or H // heads, intermediate=hf["intermediate_size"],
            vocab=hf["vocab_size"], n_pre_layers=0, n_core_layers=hf["num_hidden_layers"],
            n_post_layers=0, stages=int(hf["total_ut_steps"]),
            rope_theta=float(rope if rope is not None else hf.get("rope_theta", 10000.0)),
            rms_eps=float(hf.get("rms_norm_eps", 1e-6)),
            tie_embeddings=bool(hf.get("tie_word_embeddings", False)))
    if mt != "huginn_raven":
        raise ValueError(f"unsupported recurrent model type: {mt}")
    noise = hf.get("test_time_noise", 0)
    if isinstance(noise, bool) or not isinstance(noise, (int, float)) or float(noise) != 0.0:
        raise ValueError(f"Raven serving does not support test_time_noise; got {noise!r}")
    H, heads = hf["n_embd"], hf["n_heads"]
    hd = hf.get("head_dim") or H // heads
    layout = "olmo_post" if hd == 128 else "raven_pre"
    theta = rope if rope is not None else hf.get("rope_theta", hf.get("rope_base"))
    if theta is None:
        raise ValueError("Raven config requires a RoPE base")
    init = hf.get("init_values") or {}
    return ModelConfig(
        name=name or "raven", family="raven", layout=layout, hidden=H, n_heads=heads,
        n_kv_heads=hf.get("num_key_value_heads") or heads, head_dim=hd,
        intermediate=hf["intermediate_size"], vocab=hf["vocab_size"],
        n_pre_layers=hf["n_layers_in_prelude"], n_core_layers=hf["n_layers_in_recurrent_block"],
        n_post_layers=hf["n_layers_in_coda"], stages=int(hf["mean_recurrence"]),
        rope_theta=float(theta), rms_eps=float(hf.get("norm_eps", 1e-6)),
        embed_scale=float(init.get("embed_scale", math.sqrt(H))),
        init_std=float(init.get("std", math.sqrt(2 / (5 * H)))),
        qk_norm=layout == "olmo_post", adapter_bias=bool(hf.get("bias", False)),
        tie_embeddings=bool(hf.get("tie_embeddings", False)))


def get_config(name: str, **overrides) -> ModelConfig:
    cfg = PRESETS[name]
    return replace(cfg, **overrides) if overrides else cfg


def parse_loopspec_flags(stages: int, first: int, second: int | None):
    """CLI semantics of `--loopspec --first K [--second D]` (server/cli.py:88-96,162-168).

    D must be a multiple of K; returns (K, X) with X = D // K, validated by
    PipelineSchedule (K | S, K < S, 1 < X < S/K).
    """
    if first <= 0:
        raise ValueError("--first must be positive")
    if second is None:
        return first, None
    if second % first:
        raise ValueError("--second must be a multiple of --first")
    if second <= first:
        raise ValueError("--second must be greater than --first")
    return first, second // first
