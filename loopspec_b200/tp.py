"""Tensor parallelism over NVLink: one process per GPU, one shard per rank.

Each rank runs a narrow engine: 1/T of the attention heads (q, k and v rows
of its heads, the matching o_proj columns, KV cache of its heads) and 1/T of
the MLP columns (gate and up rows, the matching down_proj columns); the
embedding, adapter, norms outside attention and the lm_head stay whole on
every rank. The O and down projections of each layer then hold partial sums
that the engine's residual kernel adds over all ranks, and OLMo2's QK-norm
adds the ranks' sums of squares, through memory the ranks map from each other
(CUDA IPC, P2P loads over NVLink) and in rank order, so every rank computes
the same rows, logits and decisions and the host loops need no communication
after start-up. The reference has no tensor parallelism for LoopSpec
(cli.py:97-108 rejects it); the parity target is TP-N greedy output equal to
the TP-1 output.
"""

from __future__ import annotations

import dataclasses
from typing import Callable

from .config import ModelConfig

_QKV = "self_attn.qkv_proj.weight"
_O = "self_attn.o_proj.weight"
_GU = "mlp.gate_up_proj.weight"
_DOWN = "mlp.down_proj.weight"
_QN = "self_attn.q_norm.weight"
_KN = "self_attn.k_norm.weight"


def check_divisible(cfg: ModelConfig, ranks: int) -> None:
    if ranks < 1 or cfg.n_kv_heads % ranks or cfg.n_heads % ranks or cfg.intermediate % ranks:
        raise ValueError(f"{cfg.name}: {ranks} ranks must divide n_heads ({cfg.n_heads}), "
                         f"n_kv_heads ({cfg.n_kv_heads}) and intermediate ({cfg.intermediate})")


def shard_config(cfg: ModelConfig, ranks: int) -> ModelConfig:
    """The per-rank model: heads, KV heads and MLP width divided by `ranks`."""
    check_divisible(cfg, ranks)
    return dataclasses.replace(cfg, n_heads=cfg.n_heads // ranks, n_kv_heads=cfg.n_kv_heads // ranks,
                               intermediate=cfg.intermediate // ranks)


def shard_weight(name: str, t, cfg: ModelConfig, rank: int, ranks: int):
    """Rank `rank`'s part of one weight of the full model (a view or a copy)."""
    hd = cfg.head_dim
    qd, kvd = cfg.n_heads * hd, cfg.n_kv_heads * hd
    ql, kvl, il = qd // ranks, kvd // ranks, cfg.intermediate // ranks
    if name.endswith(_QKV):        # rows: q heads, then k heads, then v heads
        q, k, v = t[:qd], t[qd:qd + kvd], t[qd + kvd:]
        return _cat([q[rank * ql:(rank + 1) * ql], k[rank * kvl:(rank + 1) * kvl],
                     v[rank * kvl:(rank + 1) * kvl]])
    if name.endswith(_O):          # columns: the rank's heads
        return t[:, rank * ql:(rank + 1) * ql]
    if name.endswith(_GU):         # rows: gate, then up
        I = cfg.intermediate
        return _cat([t[rank * il:(rank + 1) * il], t[I + rank * il:I + (rank + 1) * il]])
    if name.endswith(_DOWN):       # columns: the rank's MLP width
        return t[:, rank * il:(rank + 1) * il]
    if name.endswith(_QN):
        return t[rank * ql:(rank + 1) * ql]
    if name.endswith(_KN):
        return t[rank * kvl:(rank + 1) * kvl]
    return t


def _cat(parts):
    import torch
    return torch.cat(parts, 0)


def shard_weights(weights: dict, cfg: ModelConfig, rank: int, ranks: int) -> dict:
    """Contiguous per-rank weights for the engine of shard_config(cfg, ranks)."""
    check_divisible(cfg, ranks)
    return {n: shard_weight(n, t, cfg, rank, ranks).contiguous() for n, t in weights.items()}


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """Every rank's handle bytes in rank order (torch.distributed, any backend)."""
    import torch.distributed as dist
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return [bytes(h) for h in out]


def make_tp_engine(cfg: ModelConfig, schedule, weights: dict, rank: int, ranks: int, *,
                   device: int, exchange: Callable[[bytes], list] = exchange_handles, **engine_kw):
    """Build rank `rank`'s engine from the full model's weights (on its GPU)
    and connect it to its peers. `exchange(handle)` must return every rank's
    handle in rank order; the default gathers them over torch.distributed.
    All ranks must call this together, and later make the same engine calls."""
    from .engine import Engine
    eng = Engine(shard_config(cfg, ranks), schedule, shard_weights(weights, cfg, rank, ranks),
                 device=device, **engine_kw)
    try:
        handles = exchange(eng.tp_init(rank, ranks))
        if len(handles) != ranks:
            raise ValueError(f"expected {ranks} handles, got {len(handles)}")
        eng.tp_attach(handles)
    except Exception:
        eng.close()
        raise
    eng.full_cfg = cfg
    return eng
