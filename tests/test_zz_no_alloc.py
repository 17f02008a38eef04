"""The allocation-free decode attention entry point (ls_decode_attention_noalloc).

It serves callers that cannot allocate device memory, so its scratch lives in
a fixed array inside the library. This test calls it through the C ABI twice
in a row and checks each result against the workspace entry point
(ls_decode_attention) with the attention tolerance used elsewhere (1e-4).
Collected last (file name) so a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, nh, nkv, hd, lens):
    g = torch.Generator().manual_seed(seed)
    n_slots, max_ctx = 2048, 1024
    perm = torch.randperm(n_slots, generator=g)
    m = torch.full((3, max_ctx), -1, dtype=torch.int32)
    m[0, :900] = perm[:900].to(torch.int32)
    m[1, :400] = m[0, :400]                       # row 1 forks row 0 at 400
    m[1, 400:800] = perm[900:1300].to(torch.int32)
    m[2, :300] = perm[1300:1600].to(torch.int32)
    rows = torch.tensor([i % 3 for i in range(len(lens))], dtype=torch.int32)
    lens = torch.tensor(lens, dtype=torch.int32)
    K = torch.randn(n_slots, nkv * hd, generator=g).to(torch.bfloat16)
    V = torch.randn(n_slots, nkv * hd, generator=g).to(torch.bfloat16)
    q = torch.randn(len(lens), nh * hd, generator=g)
    dev = torch.device("cuda:0")
    return [t.to(dev) for t in (q, K, V, m, rows, lens)]


def _call_noalloc(q, K, V, m, rows, lens, nh, nkv, hd, out):
    from loopspec_b200 import _lib
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    torch.cuda.synchronize()
    code = _lib.lib().ls_decode_attention_noalloc(
        p(q), p(K), p(V), p(m), p(rows), p(lens), q.shape[0], nh, nkv, hd, K.shape[0],
        m.shape[0], m.shape[1], p(out), None)
    _lib.check(code)


def test_noalloc_matches_workspace_entry_point_twice():
    from loopspec_b200.attention import decode_attention
    from loopspec_b200.build import build
    build()
    # lane i reads row i % 3: rows hold 900, 800 and 300 positions
    cases = [(16, 16, 128, [900, 800, 300, 1, 257, 299]),
             (8, 2, 64, [37, 700, 299, 900, 256])]
    for seed, (nh, nkv, hd, lens) in enumerate(cases):
        q, K, V, m, rows, lens_t = _inputs(seed, nh, nkv, hd, lens)
        torch.cuda.synchronize()
        ref = decode_attention(q, K, V, m, rows, lens_t, n_heads=nh, n_kv_heads=nkv, head_dim=hd)
        out = torch.full_like(ref, float("nan"))
        _call_noalloc(q, K, V, m, rows, lens_t, nh, nkv, hd, out)
        torch.testing.assert_close(out, ref, atol=1e-4, rtol=1e-4)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from loopspec_b200._lib import LS_ECAPACITY, EngineError
    from loopspec_b200.attention import noalloc_limit
    from loopspec_b200.build import build
    build()
    assert noalloc_limit() == 4 << 20
    nh, nkv, hd = 32, 16, 128           # 32 heads x 32 chunks x 128 dims x 4 B = 512 KiB per lane
    q, K, V, m, rows, lens = _inputs(5, nh, nkv, hd, [10] * 16)
    big_map = torch.full((3, 8192), -1, dtype=torch.int32, device=q.device)
    big_map[:, :1024] = m
    out = torch.empty(16, nh * hd, device=q.device)
    with pytest.raises(EngineError) as err:
        _call_noalloc(q, K, V, big_map, rows, lens, nh, nkv, hd, out)
    assert err.value.code == LS_ECAPACITY
