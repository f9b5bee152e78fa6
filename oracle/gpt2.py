"""ORACLE (test infrastructure): CPU restatement of the reference GPT-2 forward.

Follows `GPT2Model.forward` (examples/gpt2/model.py:845-1112) on its "gpu"
backend, using the formulas of the reference's GPU kernels on CPU tensors:

  embedding   bf16(wte[ids] + wpe[pos])                           model.py:866-876
  layernorm   bf16((x32 - mean) / sqrt(var + eps) * g32 + b32)    kernels/layernorm.py:24-48
  linear      bf16(x32 @ W32) with W the Conv1D [in, out] weight,  model.py:640-654,
              then + bias in bf16                                   kernels/matmul.py:276-277
  attention   fp32 scores * scale, causal mask (key <= pos+s),    kernels/attention.py:27-179
              softmax in fp32, P rounded to bf16 before P@V
  GELU        tanh form in fp32, bf16 out                          kernels/gelu.py:25-45
  add         bf16(a32 + b32)                                      kernels/add.py
  LM head     x32 @ wte32^T (fp32 logits)                          model.py:1100-1112

Only tests and the CPU baseline of bench.py use this module.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .qwen import attention


def _bf(x):
    return x.to(torch.bfloat16)


def layernorm(x, g, b, eps):
    x32 = x.float()
    mean = x32.mean(-1, keepdim=True)
    xc = x32 - mean
    var = (xc * xc).mean(-1, keepdim=True)
    return _bf(xc / torch.sqrt(var + eps) * g.float() + b.float())


def conv1d(x, w, b):
    """HF Conv1D: x @ w ([in, out]) + b, rounded as the reference's linear does."""
    return _bf(x.float() @ w.float()) + b


def gelu_tanh(x):
    return _bf(F.gelu(x.float(), approximate="tanh"))


class OracleGPT2:
    """Restated forward over a state dict of bf16 CPU tensors."""

    def __init__(self, sd, cfg):
        self.cfg = cfg
        self.sd = sd

    def new_cache(self, batch, max_seq):
        c = self.cfg
        shape = (batch, c.n_head, max_seq, c.head_dim)
        return {"k": [torch.zeros(shape, dtype=torch.bfloat16) for _ in range(c.n_layer)],
                "v": [torch.zeros(shape, dtype=torch.bfloat16) for _ in range(c.n_layer)], "len": 0}

    @torch.no_grad()
    def forward(self, ids, cache):
        c, sd = self.cfg, self.sd
        B, S = ids.shape
        pos = cache["len"]
        H, HD, D, eps = c.n_head, c.head_dim, c.n_embd, c.ln_eps
        positions = torch.arange(pos, pos + S)
        x = _bf(sd["transformer.wte.weight"][ids].float() + sd["transformer.wpe.weight"][positions].float())
        for i in range(c.n_layer):
            p = f"transformer.h.{i}"
            xn = layernorm(x, sd[f"{p}.ln_1.weight"], sd[f"{p}.ln_1.bias"], eps)
            qkv = conv1d(xn, sd[f"{p}.attn.c_attn.weight"], sd[f"{p}.attn.c_attn.bias"])
            q, k, v = qkv.split(D, dim=-1)
            q = q.reshape(B, S, H, HD).transpose(1, 2)
            cache["k"][i][:, :, pos:pos + S] = k.reshape(B, S, H, HD).transpose(1, 2)
            cache["v"][i][:, :, pos:pos + S] = v.reshape(B, S, H, HD).transpose(1, 2)
            o = attention(q, cache["k"][i][:, :, :pos + S], cache["v"][i][:, :, :pos + S], pos,
                          1.0 / math.sqrt(HD))
            o = o.transpose(1, 2).reshape(B, S, D)
            a = conv1d(o, sd[f"{p}.attn.c_proj.weight"], sd[f"{p}.attn.c_proj.bias"])
            x = _bf(x.float() + a.float())
            xn = layernorm(x, sd[f"{p}.ln_2.weight"], sd[f"{p}.ln_2.bias"], eps)
            h = gelu_tanh(conv1d(xn, sd[f"{p}.mlp.c_fc.weight"], sd[f"{p}.mlp.c_fc.bias"]))
            m = conv1d(h, sd[f"{p}.mlp.c_proj.weight"], sd[f"{p}.mlp.c_proj.bias"])
            x = _bf(x.float() + m.float())
        cache["len"] = pos + S
        x = layernorm(x, sd["transformer.ln_f.weight"], sd["transformer.ln_f.bias"], eps)
        return x.float() @ sd["transformer.wte.weight"].float().t()  # [B, S, V] fp32

    def generate(self, ids, max_new_tokens):
        B, S = ids.shape
        cache = self.new_cache(B, S + max_new_tokens)
        logits = self.forward(ids, cache)[:, -1]
        out = [logits.argmax(-1)]
        for _ in range(max_new_tokens - 1):
            logits = self.forward(out[-1].view(B, 1), cache)[:, -1]
            out.append(logits.argmax(-1))
        return torch.stack(out, 1)
