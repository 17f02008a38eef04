"""Tensor-parallel host logic on CPU: the shard layout, the per-layer exchange
algebra the engine implements (O / down partials and QK-norm sums added over
ranks), and the handle exchange over torch.distributed (gloo, 2 ranks)."""

import dataclasses
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from loopspec_b200.config import get_config
from loopspec_b200.tp import check_divisible, exchange_handles, make_tp_engine, shard_config, shard_weights
from loopspec_b200.weights import init_random_weights


def test_shard_config_divides_heads_and_mlp():
    cfg = get_config("raven-olmo")
    for t in (2, 4, 8):
        c = shard_config(cfg, t)
        assert (c.n_heads, c.n_kv_heads, c.intermediate) == (cfg.n_heads // t, cfg.n_kv_heads // t,
                                                             cfg.intermediate // t)
        assert (c.hidden, c.head_dim, c.vocab) == (cfg.hidden, cfg.head_dim, cfg.vocab)
    with pytest.raises(ValueError):
        check_divisible(cfg, 3)


@pytest.mark.parametrize("name,ranks", [("tiny-raven-olmo", 2), ("tiny-raven-llama", 1), ("tiny", 2),
                                        ("tiny", 4)])
def test_shards_reassemble_the_full_weights(name, ranks):
    cfg = get_config(name)
    full = init_random_weights(cfg, 0, dtype=torch.float32)
    shards = [shard_weights(full, cfg, r, ranks) for r in range(ranks)]
    hd = cfg.head_dim
    qd, kvd, I = cfg.n_heads * hd, cfg.n_kv_heads * hd, cfg.intermediate
    ql, kvl, il = qd // ranks, kvd // ranks, I // ranks
    for n, t in full.items():
        parts = [s[n] for s in shards]
        if n.endswith("qkv_proj.weight"):
            q = torch.cat([p[:ql] for p in parts])
            k = torch.cat([p[ql:ql + kvl] for p in parts])
            v = torch.cat([p[ql + kvl:] for p in parts])
            assert torch.equal(torch.cat([q, k, v]), t)
        elif n.endswith("gate_up_proj.weight"):
            g = torch.cat([p[:il] for p in parts])
            u = torch.cat([p[il:] for p in parts])
            assert torch.equal(torch.cat([g, u]), t)
        elif n.endswith("o_proj.weight") or n.endswith("down_proj.weight"):
            assert torch.equal(torch.cat(parts, 1), t)
        elif n.endswith("q_norm.weight") or n.endswith("k_norm.weight"):
            assert torch.equal(torch.cat(parts), t)
        else:
            assert all(torch.equal(p, t) for p in parts)
        assert all(p.is_contiguous() for p in parts)
    # the shard has exactly the narrow model's shapes
    from loopspec_b200.weights import weight_shapes
    narrow = weight_shapes(shard_config(cfg, ranks))
    assert {n: tuple(t.shape) for n, t in shards[0].items()} == narrow


# -- one OLMo2 post-norm layer with QK-norm, float64, S causal positions -----

def _rms(x, w, eps):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w


def _rope(x, pos, theta, hd):
    half = hd // 2
    inv = theta ** (-torch.arange(half, dtype=torch.float64) * 2 / hd)
    ang = pos[:, None].double() * inv[None]
    c, s = torch.cos(ang)[:, None], torch.sin(ang)[:, None]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def _attention(q, k, v, nh, nkv, hd):
    S = q.shape[0]
    q, k, v = q.view(S, nh, hd), k.view(S, nkv, hd), v.view(S, nkv, hd)
    g = nh // nkv
    k, v = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
    sc = torch.einsum("shd,thd->hst", q, k) / math.sqrt(hd)
    sc = sc.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
    return torch.einsum("hst,thd->shd", sc.softmax(-1), v).reshape(S, nh * hd)


def _layer_partials(x, W, p, cfg, nh, nkv, I, qk_sums):
    """One rank's attention and MLP partials (dense when it holds all heads).
    qk_sums(ssq, ssk) -> the sums of squares over every rank."""
    hd, eps = cfg.head_dim, cfg.rms_eps
    pos = torch.arange(x.shape[0])
    qkv = x @ W[p + "self_attn.qkv_proj.weight"].T
    qd, kd = nh * hd, nkv * hd
    q, k, v = qkv[:, :qd], qkv[:, qd:qd + kd], qkv[:, qd + kd:]
    ssq, ssk = qk_sums((q * q).sum(-1, keepdim=True), (k * k).sum(-1, keepdim=True))
    q = q / torch.sqrt(ssq / (cfg.n_heads * hd) + eps) * W[p + "self_attn.q_norm.weight"]
    k = k / torch.sqrt(ssk / (cfg.n_kv_heads * hd) + eps) * W[p + "self_attn.k_norm.weight"]
    q = _rope(q.view(-1, nh, hd), pos, cfg.rope_theta, hd).reshape(-1, qd)
    k = _rope(k.view(-1, nkv, hd), pos, cfg.rope_theta, hd).reshape(-1, kd)
    o_part = _attention(q, k, v, nh, nkv, hd) @ W[p + "self_attn.o_proj.weight"].T
    return o_part


def _mlp_partial(r, W, p, I):
    gu = r @ W[p + "mlp.gate_up_proj.weight"].T
    return (torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]) @ W[p + "mlp.down_proj.weight"].T


@pytest.mark.parametrize("ranks", [2, 4])
def test_sharded_olmo_layer_equals_dense_layer(ranks):
    # OLMo2 post-norm block with QK-norm (the layout of config 5), GQA 8:4
    cfg = dataclasses.replace(get_config("tiny-raven-olmo"), hidden=64, n_heads=8, n_kv_heads=4,
                              head_dim=16, intermediate=96)
    W = {n: t.double() for n, t in init_random_weights(cfg, 3, dtype=torch.float32, std=0.2).items()}
    for n in W:
        if n.endswith("norm.weight"):
            W[n] = 1 + 0.1 * torch.randn(W[n].shape, dtype=torch.float64, generator=torch.Generator().manual_seed(7))
    p, eps = "recurrent_executor.blocks.0.", cfg.rms_eps
    x = torch.randn(6, cfg.hidden, dtype=torch.float64, generator=torch.Generator().manual_seed(1))

    def block(o_sum, mlp_sum):
        r = x + _rms(o_sum, W[p + "post_attention_layernorm.weight"], eps)
        return r, lambda m: r + _rms(m, W[p + "post_feedforward_layernorm.weight"], eps)

    # dense
    o = _layer_partials(x, W, p, cfg, cfg.n_heads, cfg.n_kv_heads, cfg.intermediate, lambda a, b: (a, b))
    r, fin = block(o, None)
    dense = fin(_mlp_partial(r, W, p, cfg.intermediate))

    # tensor parallel: partial sums of squares and partial O / down rows added over ranks
    c = shard_config(cfg, ranks)
    sh = [shard_weights(W, cfg, t, ranks) for t in range(ranks)]
    hd = cfg.head_dim
    sums = []
    for t in range(ranks):
        qkv = x @ sh[t][p + "self_attn.qkv_proj.weight"].T
        q, k = qkv[:, :c.n_heads * hd], qkv[:, c.n_heads * hd:(c.n_heads + c.n_kv_heads) * hd]
        sums.append(((q * q).sum(-1, keepdim=True), (k * k).sum(-1, keepdim=True)))
    tot = (sum(s[0] for s in sums), sum(s[1] for s in sums))
    o_tp = sum(_layer_partials(x, sh[t], p, cfg, c.n_heads, c.n_kv_heads, c.intermediate, lambda a, b: tot)
               for t in range(ranks))
    r_tp, fin_tp = block(o_tp, None)
    tp = fin_tp(sum(_mlp_partial(r_tp, sh[t], p, c.intermediate) for t in range(ranks)))
    assert torch.allclose(tp, dense, rtol=0, atol=1e-10)


# -- handle exchange over torch.distributed (gloo) ---------------------------

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_rank(rank, ranks, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ranks)
    try:
        got = exchange_handles(bytes([rank + 1]) * 128)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_exchange_handles_returns_every_rank_in_rank_order():
    ranks, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_exchange_rank, args=(r, ranks, port, q)) for r in range(ranks)]
    for pr in procs:
        pr.start()
    res = dict(q.get(timeout=120) for _ in range(ranks))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    for r in range(ranks):
        assert res[r] == [bytes([t + 1]) * 128 for t in range(ranks)]


def test_indivisible_rank_counts_are_refused_before_any_gpu_work():
    with pytest.raises(ValueError):
        shard_weights({}, get_config("raven-olmo"), 0, 3)
