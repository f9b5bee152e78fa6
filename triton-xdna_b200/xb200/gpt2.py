"""GPT-2 forward and greedy generation on xb200 kernels.

Mirrors `GPT2Model` of the reference (examples/gpt2/model.py:431-1206) on its
GPU path ("gpu" backend):

  token + learned position embedding (bf16 add)      model.py:866-876
  per layer: layernorm -> fused QKV linear (+bias)   model.py:1026-1031, 757-760
             head split + KV-cache write             model.py:762-775
             causal multi-head attention             model.py:777-800, kernels/attention.py:27-179
             output projection (+bias), residual add model.py:829-836, 1032-1033
             layernorm, fc (+bias), tanh GELU,       model.py:1034-1059
             proj (+bias), residual add
  final layernorm, tied LM head in fp32              model.py:1082-1112
  greedy argmax generation with a KV cache           model.py:1119-1206

All four sizes (gpt2, -medium, -large, -xl) share the kernels: head_dim is 64
everywhere, hidden sizes are multiples of 8.  Hugging Face stores the
projections as Conv1D weights [in, out]; they are transposed once at load
into the [out, in] layout of the linear kernel (the reference passes
`weight.t()` to `triton_linear`, model.py:640-654).

Deliberate differences from the reference: biases are added in fp32 inside
the GEMM epilogue (the reference rounds the product to bf16 and then adds the
bias in bf16, kernels/matmul.py:276-277), the attention residual of small
batches is added inside the projection's split-K reduction, and generation is
batched (the reference's `generate` is batch 1 and stops at EOS; here every
sequence runs the requested number of steps).
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from . import ops
from .qwen import DecodeGraphs

# (n_layer, n_head, n_embd) of the four published sizes (model.py:90-108)
GPT2_SIZES = {
    "gpt2": (12, 12, 768),
    "gpt2-medium": (24, 16, 1024),
    "gpt2-large": (36, 20, 1280),
    "gpt2-xl": (48, 25, 1600),
}


@dataclass
class GPT2Config:
    """GPT-2 dimensions (model.py:86-112): vocab 50257, 1024 positions, LN eps 1e-5."""

    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    vocab_size: int = 50257
    n_positions: int = 1024
    ln_eps: float = 1e-5

    @classmethod
    def variant(cls, name: str = "gpt2") -> "GPT2Config":
        n_layer, n_head, n_embd = GPT2_SIZES[name]
        return cls(n_layer=n_layer, n_head=n_head, n_embd=n_embd)

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def n_kv_head(self) -> int:
        return self.n_head

    @property
    def mlp(self) -> int:
        return 4 * self.n_embd


def random_weights(cfg: GPT2Config, seed: int = 0, std: float = 0.02) -> dict:
    """Seeded random-init bf16 weights under the Hugging Face GPT-2 state-dict
    names the reference loads (model.py:519-563): Conv1D weights [in, out]
    and biases N(0, std), layernorm weights 1 + N(0, std), biases N(0, std),
    token embeddings N(0, std), position embeddings N(0, std / 2)."""
    g = torch.Generator().manual_seed(seed)
    D, V, P, F = cfg.n_embd, cfg.vocab_size, cfg.n_positions, cfg.mlp

    def w(*shape, base=0.0, s=std):
        return (base + s * torch.randn(shape, generator=g)).to(torch.bfloat16)

    sd = {"transformer.wte.weight": w(V, D), "transformer.wpe.weight": w(P, D, s=std / 2)}
    for i in range(cfg.n_layer):
        p = f"transformer.h.{i}"
        sd[f"{p}.ln_1.weight"] = w(D, base=1.0)
        sd[f"{p}.ln_1.bias"] = w(D)
        sd[f"{p}.attn.c_attn.weight"] = w(D, 3 * D)
        sd[f"{p}.attn.c_attn.bias"] = w(3 * D)
        sd[f"{p}.attn.c_proj.weight"] = w(D, D)
        sd[f"{p}.attn.c_proj.bias"] = w(D)
        sd[f"{p}.ln_2.weight"] = w(D, base=1.0)
        sd[f"{p}.ln_2.bias"] = w(D)
        sd[f"{p}.mlp.c_fc.weight"] = w(D, F)
        sd[f"{p}.mlp.c_fc.bias"] = w(F)
        sd[f"{p}.mlp.c_proj.weight"] = w(F, D)
        sd[f"{p}.mlp.c_proj.bias"] = w(D)
    sd["transformer.ln_f.weight"] = w(D, base=1.0)
    sd["transformer.ln_f.bias"] = w(D)
    return sd


class KVCache:
    """Per-layer K / V caches [B, n_head, max_seq, 64] (model.py:1119-1142)."""

    def __init__(self, cfg: GPT2Config, batch: int, max_seq: int, device):
        shape = (batch, cfg.n_head, max_seq, cfg.head_dim)
        self.k = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.n_layer)]
        self.v = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.n_layer)]
        self.batch = batch
        self.max_seq = max_seq
        self.length = 0


class GPT2Model:
    def __init__(self, state_dict: dict, cfg: GPT2Config | None = None, device="cuda"):
        self.cfg = cfg or GPT2Config()
        c = self.cfg
        if c.head_dim != 64 or c.n_embd % 8:
            raise ValueError("the attention kernels take head_dim 64 and rows of whole 16-byte vectors")
        self.device = torch.device(device)
        dev = self.device

        def t(name):
            return state_dict[name].to(device=dev, dtype=torch.bfloat16).contiguous()

        def conv1d(name):  # Conv1D [in, out] -> linear weight [out, in]
            return state_dict[name].to(device=dev, dtype=torch.bfloat16).t().contiguous()

        self.wte = t("transformer.wte.weight")
        self.wpe = t("transformer.wpe.weight")
        self.layers = []
        for i in range(c.n_layer):
            p = f"transformer.h.{i}"
            self.layers.append({
                "ln1_w": t(f"{p}.ln_1.weight"), "ln1_b": t(f"{p}.ln_1.bias"),
                "qkv_w": conv1d(f"{p}.attn.c_attn.weight"), "qkv_b": t(f"{p}.attn.c_attn.bias"),
                "proj_w": conv1d(f"{p}.attn.c_proj.weight"), "proj_b": t(f"{p}.attn.c_proj.bias"),
                "ln2_w": t(f"{p}.ln_2.weight"), "ln2_b": t(f"{p}.ln_2.bias"),
                "fc_w": conv1d(f"{p}.mlp.c_fc.weight"), "fc_b": t(f"{p}.mlp.c_fc.bias"),
                "mproj_w": conv1d(f"{p}.mlp.c_proj.weight"), "mproj_b": t(f"{p}.mlp.c_proj.bias"),
            })
        self.lnf_w = t("transformer.ln_f.weight")
        self.lnf_b = t("transformer.ln_f.bias")
        self.scale = 1.0 / math.sqrt(c.head_dim)
        self._chain = None  # decided at the first decode step

    def new_cache(self, batch: int, max_seq: int) -> KVCache:
        if max_seq > self.cfg.n_positions:
            raise ValueError(f"cache length {max_seq} exceeds the position table ({self.cfg.n_positions})")
        return KVCache(self.cfg, batch, max_seq, self.device)

    def _chain_ok(self) -> bool:
        """Decode steps run as decode chains (one launch per block besides its
        attention) when XB_DECODE_CHAIN=1 (or use_decode_chain(True)) and every
        linear fits one (not gpt2-xl's mlp c_proj, K = 6400); otherwise as
        single-launch decode linears."""
        if self._chain is None:
            self.use_decode_chain(os.environ.get("XB_DECODE_CHAIN", "0") == "1")
        return self._chain

    def use_decode_chain(self, on: bool) -> bool:
        """Choose the decode-chain path for later decode steps (if the shapes
        allow it); returns whether it is used."""
        self._chain = bool(on) and self.cfg.mlp <= ops.CHAIN_MAX_K
        return self._chain

    def _decode_chain_layers(self, x, xin, cache, pos: int, q_buf, attn):
        """The blocks of one decode step: per block, the attention kernel and
        one decode chain -- attn c_proj + residual (with the statistics of
        ln_2), c_fc + GELU (ln_2 applied as its input is loaded), mlp c_proj
        + residual, and the next block's c_attn + head split + KV write (its
        ln_1 applied the same way).  The first block's c_attn is a chain of
        its own (examples/gpt2/model.py:1032-1059 per block)."""
        c = self.cfg
        M, D = x.shape
        H, HD, eps = c.n_head, c.head_dim, c.ln_eps
        dev = self.device
        y = torch.empty((M, D), dtype=torch.bfloat16, device=dev)
        h = torch.empty((M, c.mlp), dtype=torch.bfloat16, device=dev)
        xs = [x, torch.empty((M, D), dtype=torch.bfloat16, device=dev)]  # residual stream, ping-pong
        st_post = ops.decode_stats(D, dev)
        st_in = ops.decode_stats(D, dev)
        sync = ops.decode_chain_sync(dev)  # this workspace slot's counters

        def qkv(i, xsrc, xnorm):
            L = self.layers[i]
            return ops.chain_rope_kv(xsrc, L["qkv_w"], L["qkv_b"], None, None, q_buf, cache.k[i], cache.v[i],
                                     H, H, HD, pos, xnorm=xnorm)

        phases = [qkv(0, xin, None)]
        for i, L in enumerate(self.layers):
            ops.decode_chain(phases, sync)
            ops.attention(q_buf, cache.k[i], cache.v[i], attn, M, 1, H, H, HD, pos, self.scale)
            last = i + 1 == len(self.layers)
            xr, xo = xs[i % 2], xs[(i + 1) % 2]
            phases = [
                ops.chain_residual(attn, L["proj_w"], L["proj_b"], xr, y, st_post, "layer"),
                ops.chain_store(y, L["fc_w"], L["fc_b"], h, act="gelu_tanh",
                                xnorm=(st_post, L["ln2_w"], L["ln2_b"], eps, "layer")),
                ops.chain_residual(h, L["mproj_w"], L["mproj_b"], y, xo, None if last else st_in,
                                   None if last else "layer"),
            ]
            if not last:
                nxt = self.layers[i + 1]
                phases.append(qkv(i + 1, xo, (st_in, nxt["ln1_w"], nxt["ln1_b"], eps, "layer")))
        ops.decode_chain(phases, sync)
        return xs[len(self.layers) % 2]

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, cache: KVCache, last_only: bool = False,
                next_token: torch.Tensor | None = None) -> torch.Tensor | None:
        """ids [B, S] int64 on the device; appends S positions to `cache`.
        Returns fp32 logits [B, S, vocab], or [B, vocab] of the last position;
        with `next_token` (int64 [B]) it writes the greedy token of the last
        position there instead (LM head and argmax in one pass, no logits)
        and returns None."""
        c = self.cfg
        B, S = ids.shape
        if cache.batch != B:
            raise ValueError("cache batch size differs from the input")
        pos = cache.length
        if pos + S > cache.max_seq:
            raise ValueError("KV cache full")
        M = B * S
        D, H, HD = c.n_embd, c.n_head, c.head_dim
        x = ops.embedding_pos(self.wte, self.wpe, ids, pos).reshape(M, D)
        q_buf = torch.empty((B, H, S, HD), dtype=torch.bfloat16, device=self.device)
        attn = torch.empty((M, D), dtype=torch.bfloat16, device=self.device)
        # decode step: each linear is one launch that also does what follows it
        # (head split + KV write; residual add + the row statistics of the next
        # layernorm, which the next linear applies as it loads its input)
        decode = S == 1 and M <= ops.SMALL_M
        if decode:
            xin, xnorm = ops.layernorm(x, self.layers[0]["ln1_w"], self.layers[0]["ln1_b"], c.ln_eps), None
        chain = decode and self._chain_ok()
        if chain:
            x = self._decode_chain_layers(x, xin, cache, pos, q_buf, attn)
        for i, L in enumerate(self.layers if not chain else ()):
            if decode:
                ops.decode_linear_rope_kv(xin, L["qkv_w"], L["qkv_b"], None, None, q_buf, cache.k[i], cache.v[i],
                                          H, H, HD, pos, xnorm=xnorm)
            else:
                xn = ops.layernorm(x, L["ln1_w"], L["ln1_b"], c.ln_eps)
                # c_attn GEMM with the head split + KV write in its epilogue
                ops.linear_qkv_rope(xn, L["qkv_w"], L["qkv_b"], None, None, q_buf, cache.k[i], cache.v[i],
                                    B, S, H, H, HD, pos)
            ops.attention(q_buf, cache.k[i], cache.v[i], attn, B, S, H, H, HD, pos, self.scale)
            if decode:
                y, st = ops.decode_linear_residual(attn, L["proj_w"], L["proj_b"], x, stats_kind="layer")
                h = ops.decode_linear(y, L["fc_w"], L["fc_b"], act="gelu_tanh",
                                      xnorm=(st, L["ln2_w"], L["ln2_b"], c.ln_eps, "layer"))  # ln_2 + c_fc + GELU
                last = i + 1 == len(self.layers)
                x, st = ops.decode_linear_residual(h, L["mproj_w"], L["mproj_b"], y,
                                                   stats_kind=None if last else "layer")
                if not last:
                    nxt = self.layers[i + 1]
                    xin, xnorm = x, (st, nxt["ln1_w"], nxt["ln1_b"], c.ln_eps, "layer")
                continue
            x = ops.linear(attn, L["proj_w"], L["proj_b"], residual=x)  # c_proj + residual add
            xn = ops.layernorm(x, L["ln2_w"], L["ln2_b"], c.ln_eps)
            h = ops.linear(xn, L["fc_w"], L["fc_b"], act="gelu_tanh")  # c_fc + tanh GELU, one launch
            x = ops.linear(h, L["mproj_w"], L["mproj_b"], residual=x)  # mlp c_proj + residual add
        cache.length = pos + S
        if last_only and not decode:
            x = x.reshape(B, S, D)[:, -1, :]  # strided rows: the norm kernel gathers them
        x = ops.layernorm(x, self.lnf_w, self.lnf_b, c.ln_eps,
                          out=torch.empty((x.shape[0], D), dtype=torch.bfloat16, device=self.device))
        if next_token is not None:
            if not last_only:
                raise ValueError("next_token needs last_only=True")
            ops.linear_argmax(x, self.wte, out=next_token)
            return None
        logits = ops.linear(x, self.wte, out_dtype=torch.float32)
        return logits if last_only else logits.reshape(B, S, c.vocab_size)

    @torch.no_grad()
    def generate(self, ids: torch.Tensor, max_new_tokens: int, cache: KVCache | None = None,
                 graphs: DecodeGraphs | None = None):
        """Greedy decoding (model.py:1144-1206), batched.  Returns (tokens
        [B, max_new_tokens] int64 on the device, timing dict with CUDA-event
        prefill / decode milliseconds)."""
        B, S = ids.shape
        if graphs is not None:
            cache, toks = graphs.cache, graphs.toks
            if (graphs.batch, graphs.prompt, graphs.new) != (B, S, max_new_tokens):
                raise ValueError("decode graphs were captured for another shape")
        else:
            if cache is None:
                cache = self.new_cache(B, S + max_new_tokens)
            toks = torch.empty((max_new_tokens, B), dtype=torch.int64, device=self.device)
        cache.length = 0
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        self.forward(ids, cache, last_only=True, next_token=toks[0])
        e1.record()
        if graphs is not None:
            graphs.replay()
        else:
            for step in range(1, max_new_tokens):
                self.forward(toks[step - 1].view(B, 1), cache, last_only=True, next_token=toks[step])
        e2.record()
        torch.cuda.synchronize()
        return toks.t(), {"prefill_ms": e0.elapsed_time(e1), "decode_ms": e1.elapsed_time(e2)}

    @torch.no_grad()
    def decode_graphs(self, batch: int, prompt: int, new: int, groups: int = 1) -> DecodeGraphs:
        return DecodeGraphs(self, batch, prompt, new, groups)
