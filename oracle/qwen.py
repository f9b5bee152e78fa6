"""ORACLE (test infrastructure): CPU restatement of the reference Qwen2.5 forward.

Follows `Qwen2Model.forward` (examples/qwen2_5/model.py:903-1108) on its GPU
path, using the formulas of the reference's GPU kernels and PyTorch
fallbacks, on CPU tensors:

  embedding      x = embed[ids]                                       model.py:911
  rmsnorm        bf16(x32 * rsqrt(mean(x32^2) + eps) * w32)           kernels/rmsnorm.py:29-56, model.py:761-765
  linear         bf16(x32 @ W32^T), then + bias in bf16               kernels/matmul.py:196-229, 290-291
  RoPE           bf16(q32*cos + rotate_half(q32)*sin)                 kernels/rope.py:44-67
  attention      fp32 scores * scale, causal mask (key <= pos+s),     kernels/attention.py:27-122
                 softmax in fp32, P rounded to bf16 before P@V
  add            bf16(a32 + b32)                                      kernels/add.py:20-35
  swiglu         bf16(silu(g32) * u32)                                kernels/swiglu.py:29-50
  LM head        x32 @ embed32^T (fp32 logits)                        model.py:1103-1104

GQA: each query head h reads KV head h // (n_head / n_kv_head), which is what
`repeat_interleave` over the KV heads produces (model.py:868-875).
Only tests and the CPU baseline of bench.py use this module.
"""

from __future__ import annotations

import math

import torch


def _bf(x):
    return x.to(torch.bfloat16)


def rmsnorm(x, w, eps):
    x32 = x.float()
    var = (x32 * x32).mean(-1, keepdim=True)
    return _bf(x32 * torch.rsqrt(var + eps) * w.float())


def linear(x, w, b=None):
    y = _bf(x.float() @ w.float().t())
    if b is not None:
        y = y + b  # bf16 + bf16, as the reference adds the bias after the bf16 GEMM
    return y


def rope_tables(head_dim, max_seq_len, base):
    half = head_dim // 2
    inv_freq = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) / half))
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def _rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat([-x[..., half:], x[..., :half]], dim=-1)


def apply_rope(x, cos, sin, pos):
    S = x.shape[-2]
    c = cos[pos:pos + S].view(1, 1, S, -1)
    s = sin[pos:pos + S].view(1, 1, S, -1)
    x32 = x.float()
    return _bf(x32 * c + _rotate_half(x32) * s)


def attention(q, k_all, v_all, pos, scale):
    """q [B, H, S, D]; k_all / v_all [B, KVH, T, D] (T = pos + S)."""
    B, H, S, D = q.shape
    KVH = k_all.shape[1]
    rep = H // KVH
    k = k_all.repeat_interleave(rep, dim=1).float()
    v = v_all.repeat_interleave(rep, dim=1).float()
    s = (q.float() @ k.transpose(-1, -2)) * scale  # [B, H, S, T]
    T = k.shape[2]
    qpos = pos + torch.arange(S).view(S, 1)
    kpos = torch.arange(T).view(1, T)
    s = s.masked_fill(kpos > qpos, float("-inf"))
    m = s.amax(-1, keepdim=True)
    p = torch.exp(s - m)
    l = p.sum(-1, keepdim=True)
    o = (_bf(p).float() @ v) / l
    return _bf(o)  # [B, H, S, D]


class OracleQwen:
    """Restated forward over a state dict of bf16 CPU tensors."""

    def __init__(self, sd, cfg):
        self.cfg = cfg
        self.sd = sd
        self.cos, self.sin = rope_tables(cfg.head_dim, 4096, cfg.rope_theta)

    def new_cache(self, batch, max_seq):
        c = self.cfg
        shape = (batch, c.n_kv_head, max_seq, c.head_dim)
        return {"k": [torch.zeros(shape, dtype=torch.bfloat16) for _ in range(c.n_layer)],
                "v": [torch.zeros(shape, dtype=torch.bfloat16) for _ in range(c.n_layer)], "len": 0}

    @torch.no_grad()
    def forward(self, ids, cache):
        c, sd = self.cfg, self.sd
        B, S = ids.shape
        pos = cache["len"]
        H, KVH, HD, D = c.n_head, c.n_kv_head, c.head_dim, c.n_embd
        x = sd["model.embed_tokens.weight"][ids]  # [B, S, D] bf16
        for i in range(c.n_layer):
            p = f"model.layers.{i}"
            xn = rmsnorm(x, sd[f"{p}.input_layernorm.weight"], c.rms_eps)
            wqkv = torch.cat([sd[f"{p}.self_attn.q_proj.weight"], sd[f"{p}.self_attn.k_proj.weight"],
                              sd[f"{p}.self_attn.v_proj.weight"]], 0)
            bqkv = torch.cat([sd[f"{p}.self_attn.q_proj.bias"], sd[f"{p}.self_attn.k_proj.bias"],
                              sd[f"{p}.self_attn.v_proj.bias"]], 0)
            qkv = linear(xn, wqkv, bqkv)
            q, k, v = qkv.split([H * HD, KVH * HD, KVH * HD], dim=-1)
            q = q.reshape(B, S, H, HD).transpose(1, 2)
            k = k.reshape(B, S, KVH, HD).transpose(1, 2)
            v = v.reshape(B, S, KVH, HD).transpose(1, 2)
            q = apply_rope(q, self.cos, self.sin, pos)
            k = apply_rope(k, self.cos, self.sin, pos)
            cache["k"][i][:, :, pos:pos + S] = k
            cache["v"][i][:, :, pos:pos + S] = v
            kf = cache["k"][i][:, :, :pos + S]
            vf = cache["v"][i][:, :, :pos + S]
            o = attention(q, kf, vf, pos, 1.0 / math.sqrt(HD))
            o = o.transpose(1, 2).reshape(B, S, H * HD)
            x = _bf(x.float() + linear(o, sd[f"{p}.self_attn.o_proj.weight"]).float())
            xn = rmsnorm(x, sd[f"{p}.post_attention_layernorm.weight"], c.rms_eps)
            g = linear(xn, sd[f"{p}.mlp.gate_proj.weight"]).float()
            u = linear(xn, sd[f"{p}.mlp.up_proj.weight"]).float()
            h = _bf(g * torch.sigmoid(g) * u)
            x = _bf(x.float() + linear(h, sd[f"{p}.mlp.down_proj.weight"]).float())
        cache["len"] = pos + S
        x = rmsnorm(x, sd["model.norm.weight"], c.rms_eps)
        return x.float() @ sd["model.embed_tokens.weight"].float().t()  # [B, S, V] fp32

    def generate(self, ids, max_new_tokens):
        B, S = ids.shape
        cache = self.new_cache(B, S + max_new_tokens)
        out = []
        logits = self.forward(ids, cache)
        tok = logits[:, -1].argmax(-1)
        out.append(tok)
        for _ in range(max_new_tokens - 1):
            logits = self.forward(tok.view(B, 1), cache)
            tok = logits[:, -1].argmax(-1)
            out.append(tok)
        return torch.stack(out, 1)
