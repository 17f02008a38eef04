"""The timeline-aware paged decode attention kernel (ls_decode_attention) vs a
torch fp32 reference of the same op, on forked timelines sharing KV slots.

Tolerance: 1e-4 abs + 1e-4 rel (fp32 softmax/accumulation; K/V are bf16 on
both sides).
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _build():
    from loopspec_b200.build import build
    build()


def make_timelines(n_slots=4096, max_ctx=1024, seed=0):
    """Row 0: 800 positions; row 1 forks row 0 at 500, row 2 forks row 1 at 600."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n_slots, generator=g)
    m = torch.full((4, max_ctx), -1, dtype=torch.int32)
    m[0, :800] = perm[:800].to(torch.int32)
    m[1, :500] = m[0, :500]
    m[1, 500:700] = perm[800:1000].to(torch.int32)
    m[2, :600] = m[1, :600]
    m[2, 600:650] = perm[1000:1050].to(torch.int32)
    m[3, :1024] = perm[2000:3024].to(torch.int32)
    lanes = [(0, 800), (1, 700), (2, 650), (0, 1), (1, 256), (2, 257), (3, 1024), (0, 255)]
    return m, lanes


def reference(q, K, V, m, lanes, nh, nkv, hd):
    out = []
    for i, (row, n) in enumerate(lanes):
        slots = m[row, :n].long()
        k = K[slots].float().view(n, nkv, hd).repeat_interleave(nh // nkv, dim=1)
        v = V[slots].float().view(n, nkv, hd).repeat_interleave(nh // nkv, dim=1)
        qi = q[i].view(nh, hd)
        s = torch.einsum("hd,nhd->hn", qi, k) / math.sqrt(hd)
        out.append(torch.einsum("hn,nhd->hd", torch.softmax(s, -1), v).reshape(-1))
    return torch.stack(out)


@pytest.mark.parametrize("nh,nkv,hd", [(16, 16, 128), (32, 8, 64), (4, 2, 128), (4, 4, 64), (8, 4, 64)])
def test_decode_attention_matches_torch(nh, nkv, hd):
    _build()
    from loopspec_b200.attention import decode_attention
    dev = torch.device("cuda:0")
    m, lanes = make_timelines()
    g = torch.Generator().manual_seed(hd + nh)
    n_slots = 4096
    K = torch.randn(n_slots, nkv * hd, generator=g).to(torch.bfloat16)
    V = torch.randn(n_slots, nkv * hd, generator=g).to(torch.bfloat16)
    q = torch.randn(len(lanes), nh * hd, generator=g)
    rows = torch.tensor([r for r, _ in lanes], dtype=torch.int32)
    lens = torch.tensor([n for _, n in lanes], dtype=torch.int32)
    ref = reference(q, K, V, m, lanes, nh, nkv, hd)
    torch.cuda.synchronize()
    out = decode_attention(q.to(dev), K.to(dev), V.to(dev), m.to(dev), rows.to(dev), lens.to(dev),
                           n_heads=nh, n_kv_heads=nkv, head_dim=hd)
    torch.testing.assert_close(out.cpu(), ref, atol=1e-4, rtol=1e-4)


def test_decode_attention_is_batch_invariant():
    _build()
    from loopspec_b200.attention import decode_attention
    dev = torch.device("cuda:0")
    m, lanes = make_timelines()
    nh, nkv, hd = 16, 16, 128
    g = torch.Generator().manual_seed(3)
    K = torch.randn(4096, nkv * hd, generator=g).to(torch.bfloat16).to(dev)
    V = torch.randn(4096, nkv * hd, generator=g).to(torch.bfloat16).to(dev)
    q = torch.randn(len(lanes), nh * hd, generator=g).to(dev)
    rows = torch.tensor([r for r, _ in lanes], dtype=torch.int32, device=dev)
    lens = torch.tensor([n for _, n in lanes], dtype=torch.int32, device=dev)
    md = m.to(dev)
    full = decode_attention(q, K, V, md, rows, lens, n_heads=nh, n_kv_heads=nkv, head_dim=hd)
    for i in range(len(lanes)):
        one = decode_attention(q[i:i + 1], K, V, md, rows[i:i + 1], lens[i:i + 1],
                               n_heads=nh, n_kv_heads=nkv, head_dim=hd)
        assert torch.equal(one[0], full[i])        # bit-identical whatever the batch


def test_decode_attention_reports_bad_indices():
    _build()
    from loopspec_b200._lib import EngineError
    from loopspec_b200.attention import decode_attention
    dev = torch.device("cuda:0")
    m, _ = make_timelines()
    K = torch.zeros(4096, 128, dtype=torch.bfloat16, device=dev)
    q = torch.zeros(1, 128, device=dev)
    rows = torch.tensor([0], dtype=torch.int32, device=dev)
    with pytest.raises(EngineError):   # position 800 of row 0 was never written (slot -1)
        decode_attention(q, K, K, m.to(dev), rows, torch.tensor([801], dtype=torch.int32, device=dev),
                         n_heads=1, n_kv_heads=1, head_dim=128)
    with pytest.raises(EngineError):   # longer than max_context
        decode_attention(q, K, K, m.to(dev), rows, torch.tensor([2000], dtype=torch.int32, device=dev),
                         n_heads=1, n_kv_heads=1, head_dim=128)
