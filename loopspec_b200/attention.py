"""Standalone branch-timeline paged decode attention (the engine's kernel).

`decode_attention` calls `ls_decode_attention` through the C ABI with raw
device pointers of torch tensors; the caller's torch tensors only provide
memory. Layout (page size 1, like the reference's SGLang pools):
  q         fp32 [n_lanes, n_heads * head_dim]   (RoPE applied)
  k_pool    bf16 [n_slots, n_kv_heads * head_dim]
  v_pool    bf16 [n_slots, n_kv_heads * head_dim]
  map       int32 [n_rows, max_context]          timeline row -> slot per position
  lane_rows int32 [n_lanes], lane_lens int32 [n_lanes]
"""

from __future__ import annotations

import ctypes

from . import _lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def workspace_bytes(n_lanes, n_heads, n_kv_heads, head_dim, max_context):
    return int(_lib.lib().ls_decode_attention_workspace_bytes(n_lanes, n_heads, n_kv_heads,
                                                              head_dim, max_context))


def decode_attention(q, k_pool, v_pool, mapping, lane_rows, lane_lens, *, n_heads, n_kv_heads,
                     head_dim, workspace=None, stream=None):
    import torch
    n = q.shape[0]
    n_rows, max_ctx = mapping.shape
    need = workspace_bytes(n, n_heads, n_kv_heads, head_dim, max_ctx)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    out = torch.empty(n, n_heads * head_dim, dtype=torch.float32, device=q.device)
    L = _lib.lib()
    code = L.ls_decode_attention(
        _ptr(q), _ptr(k_pool), _ptr(v_pool), _ptr(mapping), _ptr(lane_rows), _ptr(lane_lens), n,
        n_heads, n_kv_heads, head_dim, k_pool.shape[0], n_rows, max_ctx, _ptr(workspace),
        workspace.numel(), _ptr(out), ctypes.c_void_p(stream or 0))
    _lib.check(code)
    return out


def decode_attention_noalloc(q, k_pool, v_pool, mapping, lane_rows, lane_lens, *, n_heads,
                             n_kv_heads, head_dim, out=None, stream=None):
    """Same op without a workspace, for callers that cannot allocate device
    memory (allocator hooks, fully pre-reserved memory). The library's fixed
    scratch (`noalloc_limit()` bytes per GPU) is shared by every call on a
    device; calls that overlap on the GPU race. Pass `out` to allocate nothing
    here either."""
    import torch
    n = q.shape[0]
    n_rows, max_ctx = mapping.shape
    if out is None:
        out = torch.empty(n, n_heads * head_dim, dtype=torch.float32, device=q.device)
    L = _lib.lib()
    code = L.ls_decode_attention_noalloc(
        _ptr(q), _ptr(k_pool), _ptr(v_pool), _ptr(mapping), _ptr(lane_rows), _ptr(lane_lens), n,
        n_heads, n_kv_heads, head_dim, k_pool.shape[0], n_rows, max_ctx, _ptr(out),
        ctypes.c_void_p(stream or 0))
    _lib.check(code)
    return out


def noalloc_limit():
    return int(_lib.lib().ls_decode_attention_noalloc_limit())
