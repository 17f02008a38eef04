"""fp32 PyTorch CPU restatement of the looped-model roles (oracle, test-only).

One lane at a time, one token at a time; every attention call appends the
token's K/V to the timeline it is given and attends over the whole timeline.

Follows:
  Ouro layer (Gemma2 residual flow, Llama attention/MLP, sandwich RMSNorm)
      sglang_recurrent/modeling/ouro.py:37-82; norm mapping :28-34
  Ouro core iteration = all layers then step_norm      ouro.py:93-98
  Raven core iteration = adapter(cat(h, injected)) then core blocks
      raven.py:271-281 (RavenRecurrentExecutor.forward)
  Raven layer layouts ("raven_pre" = Llama pre-norm, "olmo_post" = OLMo2
      post-norm with QK-norm)                          contracts.py:185-197,
      raven.py:258-265,328-332
  pre role: embed * embed_scale, prelude blocks, Raven separate hidden
      components.py:117-149
  post role: coda blocks, optional final norm, lm_head components.py:175-194
Layer internals (not in the reference tree; SGLang 0.5.14): fused QKV,
neox RoPE, softmax(q k^T / sqrt(d)), O projection, SiLU(gate)*up MLP,
RMSNorm x * rsqrt(mean(x^2) + eps) * w.

Raven's recurrent hidden init: the reference draws torch RNG per pre call
(components.py:79-115), which cannot make LoopSpec equal AR because LoopSpec
runs pre once per lane. The engine keys the draw on (seed, position) with
Philox4x32-10 (Salmon et al., SC'11) and an inverse-CDF truncated normal; this
oracle restates that engine choice in `raven_initial_hidden`.
"""

from __future__ import annotations

import math

import numpy as np
import torch


def rms_norm(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope_neox(x, pos, theta):
    """x: [heads, d]; rotate the two halves (neox style). The angles are
    computed in x's precision when it is above fp32."""
    d = x.shape[-1]
    half = d // 2
    ft = torch.float64 if x.dtype == torch.float64 else torch.float32
    inv_freq = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=ft) / d))
    ang = float(pos) * inv_freq
    cos, sin = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)


# ---------------------------------------------------------------- Philox4x32-10
_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK = 0xFFFFFFFF


def philox4x32(counter, key):
    """counter: uint64 array [..., 4] of 32-bit words; key: (k0, k1)."""
    c = [counter[..., i].astype(np.uint64) for i in range(4)]
    k0, k1 = np.uint64(key[0]), np.uint64(key[1])
    for _ in range(10):
        p0 = np.uint64(_M0) * c[0]
        p1 = np.uint64(_M1) * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & np.uint64(_MASK)
        hi1, lo1 = p1 >> np.uint64(32), p1 & np.uint64(_MASK)
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
        k0 = (k0 + np.uint64(_W0)) & np.uint64(_MASK)
        k1 = (k1 + np.uint64(_W1)) & np.uint64(_MASK)
    return np.stack(c, axis=-1)


def raven_initial_hidden(seed, pos, hidden, std, embed_scale):
    """Position-keyed truncated normal(0, std) on [-3std, 3std], times embed_scale.

    Element i of position `pos` uses word i % 4 of Philox(counter=(i // 4, pos,
    0, 0), key=(seed low, seed high)); u = (w >> 8 + 0.5) / 2^24.
    """
    n4 = (hidden + 3) // 4
    ctr = np.zeros((n4, 4), dtype=np.uint64)
    ctr[:, 0] = np.arange(n4, dtype=np.uint64)
    ctr[:, 1] = np.uint64(pos)
    words = philox4x32(ctr, (seed & _MASK, (seed >> 32) & _MASK)).reshape(-1)[:hidden]
    u = ((words >> np.uint64(8)).astype(np.float64) + 0.5) / float(1 << 24)
    if std <= 0:
        return torch.zeros(hidden)
    lo = 0.5 * math.erfc(3.0 / math.sqrt(2.0))   # Phi(-3)
    p = lo + u * (1.0 - 2.0 * lo)
    x = math.sqrt(2.0) * torch.erfinv(torch.from_numpy(2.0 * p - 1.0))
    return (x * std * embed_scale).to(torch.float32)


class Timeline:
    """K/V of one (branch, role, depth) timeline: per layer, list over positions."""

    def __init__(self, n_layers):
        self.k = [[] for _ in range(n_layers)]
        self.v = [[] for _ in range(n_layers)]

    def fork(self):
        """Child timeline sharing the parent's whole current prefix (manager.py:207-232)."""
        t = Timeline(0)
        t.k = [list(x) for x in self.k]
        t.v = [list(x) for x in self.v]
        return t

    def __len__(self):
        return len(self.k[0]) if self.k else 0


class OracleModel:
    """Role forward math for one lane. `cfg` is a plain dict of config fields."""

    def __init__(self, cfg, weights, *, kv_bf16=False, dtype=torch.float32):
        """kv_bf16: store K/V in bf16 like the reference's KV pool (SGLang keeps
        the cache in the model dtype). dtype: the arithmetic precision (fp32;
        float64 measures how far two correct restatements drift apart)."""
        self.kv_bf16 = kv_bf16
        self.cfg = cfg
        self.dtype = dtype
        self.w = {k: v.detach().to(dtype).cpu() for k, v in weights.items()}
        self.family = cfg["family"]
        self.layout = cfg["layout"]
        self.H = cfg["hidden"]
        self.nh = cfg["n_heads"]
        self.nkv = cfg["n_kv_heads"]
        self.hd = cfg["head_dim"]
        self.eps = cfg["rms_eps"]
        self.theta = cfg["rope_theta"]

    # ------------------------------------------------------------------ layers
    def _attention(self, p, x, pos, tl, layer):
        w = self.w
        nh, nkv, hd = self.nh, self.nkv, self.hd
        qkv = w[p + "self_attn.qkv_proj.weight"] @ x
        q = qkv[: nh * hd]
        k = qkv[nh * hd: (nh + nkv) * hd]
        v = qkv[(nh + nkv) * hd:]
        if self.cfg.get("qk_norm"):
            q = rms_norm(q, w[p + "self_attn.q_norm.weight"], self.eps)
            k = rms_norm(k, w[p + "self_attn.k_norm.weight"], self.eps)
        q = rope_neox(q.view(nh, hd), pos, self.theta)
        k = rope_neox(k.view(nkv, hd), pos, self.theta)
        v = v.view(nkv, hd)
        if self.kv_bf16:
            # the reference's KV pool stores K (after RoPE) and V in the model dtype
            k = k.to(torch.bfloat16).to(self.dtype)
            v = v.to(torch.bfloat16).to(self.dtype)
        if len(tl.k[layer]) != pos:
            raise RuntimeError(f"timeline length {len(tl.k[layer])} != position {pos}")
        tl.k[layer].append(k)
        tl.v[layer].append(v)
        K = torch.stack(tl.k[layer])          # [L, nkv, hd]
        V = torch.stack(tl.v[layer])
        group = nh // nkv
        Kx = K.repeat_interleave(group, dim=1)  # [L, nh, hd]
        Vx = V.repeat_interleave(group, dim=1)
        scores = torch.einsum("hd,lhd->hl", q, Kx) / math.sqrt(hd)
        probs = torch.softmax(scores, dim=-1)
        out = torch.einsum("hl,lhd->hd", probs, Vx).reshape(-1)
        return w[p + "self_attn.o_proj.weight"] @ out

    def _mlp(self, p, x):
        gu = self.w[p + "mlp.gate_up_proj.weight"] @ x
        inter = gu.shape[0] // 2
        g, u = gu[:inter], gu[inter:]
        return self.w[p + "mlp.down_proj.weight"] @ (torch.nn.functional.silu(g) * u)

    def layer(self, p, h, pos, tl, layer):
        w, eps = self.w, self.eps
        if self.layout == "ouro":
            a = self._attention(p, rms_norm(h, w[p + "input_layernorm.weight"], eps), pos, tl, layer)
            r = h + rms_norm(a, w[p + "post_attention_layernorm.weight"], eps)
            m = self._mlp(p, rms_norm(r, w[p + "pre_feedforward_layernorm.weight"], eps))
            return r + rms_norm(m, w[p + "post_feedforward_layernorm.weight"], eps)
        if self.layout == "raven_pre":
            r = h + self._attention(p, rms_norm(h, w[p + "input_layernorm.weight"], eps), pos, tl, layer)
            return r + self._mlp(p, rms_norm(r, w[p + "post_attention_layernorm.weight"], eps))
        if self.layout == "olmo_post":
            r = h + rms_norm(self._attention(p, h, pos, tl, layer),
                             w[p + "post_attention_layernorm.weight"], eps)
            return r + rms_norm(self._mlp(p, r), w[p + "post_feedforward_layernorm.weight"], eps)
        raise ValueError(self.layout)

    # ------------------------------------------------------------------- roles
    def pre(self, token, pos, tl):
        """Returns (hidden, injected); injected is None for Ouro."""
        cfg = self.cfg
        h = self.w["pre_executor.embed_tokens.weight"][token] * cfg["embed_scale"]
        for i in range(cfg["n_pre_layers"]):
            h = self.layer(f"pre_executor.blocks.{i}.", h, pos, tl, i)
        if self.family == "ouro":
            return h, None
        hid = raven_initial_hidden(cfg["init_seed"], pos, self.H, cfg["init_std"], cfg["embed_scale"])
        return hid.to(self.dtype), h

    def core(self, h, injected, pos, tl):
        cfg = self.cfg
        if self.family == "raven":
            a = self.w["recurrent_executor.adapter.weight"] @ torch.cat((h, injected))
            if "recurrent_executor.adapter.bias" in self.w:
                a = a + self.w["recurrent_executor.adapter.bias"]
            h = a
        for i in range(cfg["n_core_layers"]):
            h = self.layer(f"recurrent_executor.blocks.{i}.", h, pos, tl, i)
        if self.family == "ouro":
            h = rms_norm(h, self.w["recurrent_executor.step_norm.weight"], self.eps)
        return h

    def post(self, h, pos, tl):
        cfg = self.cfg
        for i in range(cfg["n_post_layers"]):
            h = self.layer(f"post_executor.blocks.{i}.", h, pos, tl, i)
        if "post_executor.final_norm.weight" in self.w:
            h = rms_norm(h, self.w["post_executor.final_norm.weight"], self.eps)
        head = self.w.get("post_executor.lm_head.weight")
        if head is None:
            head = self.w["pre_executor.embed_tokens.weight"]
        return head @ h
