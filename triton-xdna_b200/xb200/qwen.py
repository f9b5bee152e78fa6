"""Qwen2.5 decoder forward and greedy generation on xb200 kernels.

Mirrors `Qwen2Model` of the reference (examples/qwen2_5/model.py:571-1179) on
its GPU path:

  embedding gather                                   model.py:911
  per layer: rmsnorm -> fused QKV linear (+bias)     model.py:750-765, 836-849
             RoPE + KV-cache write                   model.py:851-867, kernels/rope.py:44-67
             causal GQA attention                    model.py:868-889, kernels/attention.py:27-122
             o_proj, residual add                    model.py:893, 1045-1046
             rmsnorm, gate/up, silu*up, down, add    model.py:1047-1061
  final rmsnorm, tied LM head in fp32                model.py:1087-1106
  greedy argmax generation with a KV cache           model.py:1110-1179

Every step is an xb200 kernel (ops.*); torch only owns device memory.
Differences from the reference, all deliberate: GQA is handled natively by
the attention kernel (no repeat_interleave of K/V); the QKV bias is added in
fp32 inside the GEMM epilogue (the reference rounds the product to bf16 and
adds in bf16); generation is batched (the reference's `generate` is batch 1)
and may return last-position logits only (all a greedy step needs).
"""

from __future__ import annotations

import copy
import math
import os
import time
from dataclasses import dataclass

import torch

from . import ops


@dataclass
class QwenConfig:
    """Qwen2.5 dimensions (examples/qwen2_5/model.py:57-90)."""

    n_layer: int = 24
    n_head: int = 14
    n_kv_head: int = 2
    n_embd: int = 896
    head_dim: int = 64
    intermediate: int = 4864
    vocab_size: int = 151936
    rope_theta: float = 1000000.0
    rms_eps: float = 1e-6
    max_seq_len: int = 32768

    @classmethod
    def qwen2_5_0_5b(cls) -> "QwenConfig":
        return cls()


def random_weights(cfg: QwenConfig, seed: int = 0, std: float = 0.02) -> dict:
    """Seeded random-init bf16 weights with the HF state-dict names the
    reference loads (model.py:660-683): N(0, std) matrices and biases, RMSNorm
    weights 1 + N(0, std).  Generated on the CPU so every process (and the
    CPU oracle) gets identical weights from the same seed."""
    g = torch.Generator().manual_seed(seed)

    def w(*shape, base=0.0):
        return (base + std * torch.randn(*shape, generator=g)).to(torch.bfloat16)

    D, KV = cfg.n_embd, cfg.n_kv_head * cfg.head_dim
    sd = {"model.embed_tokens.weight": w(cfg.vocab_size, D)}
    for i in range(cfg.n_layer):
        p = f"model.layers.{i}"
        sd[f"{p}.input_layernorm.weight"] = w(D, base=1.0)
        sd[f"{p}.post_attention_layernorm.weight"] = w(D, base=1.0)
        sd[f"{p}.self_attn.q_proj.weight"] = w(cfg.n_head * cfg.head_dim, D)
        sd[f"{p}.self_attn.q_proj.bias"] = w(cfg.n_head * cfg.head_dim)
        sd[f"{p}.self_attn.k_proj.weight"] = w(KV, D)
        sd[f"{p}.self_attn.k_proj.bias"] = w(KV)
        sd[f"{p}.self_attn.v_proj.weight"] = w(KV, D)
        sd[f"{p}.self_attn.v_proj.bias"] = w(KV)
        sd[f"{p}.self_attn.o_proj.weight"] = w(D, cfg.n_head * cfg.head_dim)
        sd[f"{p}.mlp.gate_proj.weight"] = w(cfg.intermediate, D)
        sd[f"{p}.mlp.up_proj.weight"] = w(cfg.intermediate, D)
        sd[f"{p}.mlp.down_proj.weight"] = w(D, cfg.intermediate)
    sd["model.norm.weight"] = w(D, base=1.0)
    return sd


def rope_tables(head_dim: int, max_seq_len: int, base: float):
    """cos / sin tables [max_seq_len, head_dim] in fp32, computed exactly as
    examples/qwen2_5/kernels/rope.py:20-35 does."""
    half = head_dim // 2
    inv_freq = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) / half))
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


class KVCache:
    """Per-layer K / V caches [B, n_kv_head, max_seq, head_dim] (model.py:1110-1132)."""

    def __init__(self, cfg: QwenConfig, batch: int, max_seq: int, device):
        shape = (batch, cfg.n_kv_head, max_seq, cfg.head_dim)
        self.k = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.n_layer)]
        self.v = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.n_layer)]
        self.batch = batch
        self.max_seq = max_seq
        self.length = 0


class Qwen2Model:
    def __init__(self, state_dict: dict, cfg: QwenConfig | None = None, device="cuda", rope_len: int | None = None):
        self.cfg = cfg or QwenConfig()
        c = self.cfg
        self.device = torch.device(device)
        dev = self.device

        def t(name):
            return state_dict[name].to(device=dev, dtype=torch.bfloat16).contiguous()

        self.embed = t("model.embed_tokens.weight")
        self.layers = []
        for i in range(c.n_layer):
            p = f"model.layers.{i}"
            self.layers.append({
                "input_ln": t(f"{p}.input_layernorm.weight"),
                "post_ln": t(f"{p}.post_attention_layernorm.weight"),
                # fused QKV weight / bias, as model.py:840-846 builds them
                "qkv_w": torch.cat([t(f"{p}.self_attn.q_proj.weight"), t(f"{p}.self_attn.k_proj.weight"),
                                    t(f"{p}.self_attn.v_proj.weight")], 0).contiguous(),
                "qkv_b": torch.cat([t(f"{p}.self_attn.q_proj.bias"), t(f"{p}.self_attn.k_proj.bias"),
                                    t(f"{p}.self_attn.v_proj.bias")], 0).contiguous(),
                "o_w": t(f"{p}.self_attn.o_proj.weight"),
                # gate and up rows interleaved in 64-row blocks: one GEMM (or one
                # cluster split-K launch at decode) that applies silu(gate) * up
                "gate_up_w": ops.interleave_gate_up(t(f"{p}.mlp.gate_proj.weight"),
                                                    t(f"{p}.mlp.up_proj.weight")),
                "down_w": t(f"{p}.mlp.down_proj.weight"),
            })
        self.norm_w = t("model.norm.weight")
        cos, sin = rope_tables(c.head_dim, rope_len or c.max_seq_len, c.rope_theta)
        self.cos = cos.to(dev).contiguous()
        self.sin = sin.to(dev).contiguous()
        self.scale = 1.0 / math.sqrt(c.head_dim)
        self._chain = None  # decided at the first decode step

    def _chain_ok(self) -> bool:
        """Decode steps run as decode chains (one launch per layer besides its
        attention) when XB_DECODE_CHAIN=1 (or use_decode_chain(True)) and every
        linear fits one; otherwise as single-launch decode linears."""
        if self._chain is None:
            self.use_decode_chain(os.environ.get("XB_DECODE_CHAIN", "0") == "1")
        return self._chain

    def use_decode_chain(self, on: bool) -> bool:
        """Choose the decode-chain path for later decode steps (if the shapes
        allow it); returns whether it is used."""
        c = self.cfg
        self._chain = bool(on) and max(c.n_embd, c.intermediate) <= ops.CHAIN_MAX_K
        return self._chain

    def _decode_chain_layers(self, x, xin, cache: KVCache, pos: int, q_buf, attn):
        """The decoder layers of one decode step: per layer, the attention
        kernel and one decode chain -- o_proj + residual (with the statistics
        of the post-attention RMSNorm), gate/up + SwiGLU (that norm applied as
        its input is loaded), down_proj + residual, and the next layer's QKV +
        RoPE + KV write (its input norm applied the same way).  The first
        layer's QKV is a chain of its own.  Returns the residual stream after
        the last layer (examples/qwen2_5/model.py:1045-1061 per layer)."""
        c = self.cfg
        M, D = x.shape
        H, KVH, HD, eps = c.n_head, c.n_kv_head, c.head_dim, c.rms_eps
        dev = self.device
        y = torch.empty((M, D), dtype=torch.bfloat16, device=dev)
        h = torch.empty((M, c.intermediate), dtype=torch.bfloat16, device=dev)
        xs = [x, torch.empty((M, D), dtype=torch.bfloat16, device=dev)]  # residual stream, ping-pong
        st_post = ops.decode_stats(D, dev)
        st_in = ops.decode_stats(D, dev)
        sync = ops.decode_chain_sync(dev)  # this workspace slot's counters

        def qkv(i, xsrc, xnorm):
            L = self.layers[i]
            return ops.chain_rope_kv(xsrc, L["qkv_w"], L["qkv_b"], self.cos, self.sin, q_buf, cache.k[i],
                                     cache.v[i], H, KVH, HD, pos, xnorm=xnorm)

        phases = [qkv(0, xin, None)]
        for i, L in enumerate(self.layers):
            ops.decode_chain(phases, sync)
            ops.attention(q_buf, cache.k[i], cache.v[i], attn, M, 1, H, KVH, HD, pos, self.scale)
            last = i + 1 == len(self.layers)
            xr, xo = xs[i % 2], xs[(i + 1) % 2]
            phases = [
                ops.chain_residual(attn, L["o_w"], None, xr, y, st_post, "rms"),
                ops.chain_swiglu(y, L["gate_up_w"], h, xnorm=(st_post, L["post_ln"], None, eps, "rms")),
                ops.chain_residual(h, L["down_w"], None, y, xo, None if last else st_in, None if last else "rms"),
            ]
            if not last:
                phases.append(qkv(i + 1, xo, (st_in, self.layers[i + 1]["input_ln"], None, eps, "rms")))
        ops.decode_chain(phases, sync)
        return xs[len(self.layers) % 2]

    def new_cache(self, batch: int, max_seq: int) -> KVCache:
        if max_seq > self.cos.shape[0]:
            raise ValueError(f"cache length {max_seq} exceeds the RoPE table ({self.cos.shape[0]})")
        return KVCache(self.cfg, batch, max_seq, self.device)

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
        D, H, KVH, HD = c.n_embd, c.n_head, c.n_kv_head, c.head_dim
        x = ops.embedding(self.embed, ids.reshape(-1)).reshape(M, D)
        q_buf = torch.empty((B, H, S, HD), dtype=torch.bfloat16, device=self.device)
        attn = torch.empty((M, H * HD), dtype=torch.bfloat16, device=self.device)
        # decode step: each linear is one launch that also does what follows it
        # (RoPE + KV write; residual add + the row statistics of the next norm,
        # which the next linear applies as it loads its input)
        decode = S == 1 and M <= ops.SMALL_M
        if decode:
            xin, xnorm = ops.rms_norm(x, self.layers[0]["input_ln"], c.rms_eps), None
        chain = decode and self._chain_ok()
        if chain:
            x = self._decode_chain_layers(x, xin, cache, pos, q_buf, attn)
        for i, L in enumerate(self.layers if not chain else ()):
            if decode:
                ops.decode_linear_rope_kv(xin, L["qkv_w"], L["qkv_b"], self.cos, self.sin, q_buf, cache.k[i],
                                          cache.v[i], H, KVH, HD, pos, xnorm=xnorm)
            else:
                xn = ops.rms_norm(x, L["input_ln"], c.rms_eps)
                # QKV GEMM with RoPE + KV write in its epilogue
                # rope_tables() concatenates the frequencies with themselves
                ops.linear_qkv_rope(xn, L["qkv_w"], L["qkv_b"], self.cos, self.sin, q_buf, cache.k[i], cache.v[i],
                                    B, S, H, KVH, HD, pos, rope_dup=True)
            ops.attention(q_buf, cache.k[i], cache.v[i], attn, B, S, H, KVH, HD, pos, self.scale)
            if decode:
                y, st = ops.decode_linear_residual(attn, L["o_w"], None, x, stats_kind="rms")
                h = ops.decode_linear_swiglu(y, L["gate_up_w"], xnorm=(st, L["post_ln"], None, c.rms_eps, "rms"))
                last = i + 1 == len(self.layers)
                x, st = ops.decode_linear_residual(h, L["down_w"], None, y, stats_kind=None if last else "rms")
                if not last:
                    xin, xnorm = x, (st, self.layers[i + 1]["input_ln"], None, c.rms_eps, "rms")
                continue
            x = ops.linear(attn, L["o_w"], residual=x)  # o_proj + residual add (in the epilogue)
            xn = ops.rms_norm(x, L["post_ln"], c.rms_eps)
            h = ops.linear_swiglu(xn, L["gate_up_w"], interleaved=True)  # gate + up + silu*up, one GEMM
            x = ops.linear(h, L["down_w"], residual=x)  # down_proj + residual add (in the epilogue)
        cache.length = pos + S
        if last_only and not decode:
            x = x.reshape(B, S, D)[:, -1, :]  # strided rows: the norm kernel gathers them
        x = ops.rms_norm(x, self.norm_w, c.rms_eps, out=torch.empty((x.shape[0], D), dtype=torch.bfloat16,
                                                                     device=self.device))
        if next_token is not None:
            if not last_only:
                raise ValueError("next_token needs last_only=True")
            ops.linear_argmax(x, self.embed, out=next_token)
            return None
        logits = ops.linear(x, self.embed, out_dtype=torch.float32)
        return logits if last_only else logits.reshape(B, S, c.vocab_size)

    @torch.no_grad()
    def generate(self, ids: torch.Tensor, max_new_tokens: int, cache: KVCache | None = None,
                 graphs: "DecodeGraphs | None" = None):
        """Greedy decoding (model.py:1134-1179), batched.  Returns
        (tokens [B, max_new_tokens] int64 on the device, timing dict with
        CUDA-event prefill / decode milliseconds).  With `graphs` (built by
        `decode_graphs` for this cache and shape) every decode step replays a
        captured CUDA graph instead of launching its ~300 kernels from Python."""
        B, S = ids.shape
        if graphs is not None:
            cache, toks = graphs.cache, graphs.toks
            if (graphs.batch, graphs.prompt, graphs.new) != (B, S, max_new_tokens):
                raise ValueError("decode graphs were captured for another shape")
        else:
            if cache is None:
                cache = self.new_cache(B, S + max_new_tokens)
            # step-major token buffer: row `step` holds every sequence's token,
            # so the argmax writes and the next embedding reads are contiguous
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
    def decode_graphs(self, batch: int, prompt: int, new: int, groups: int = 1) -> "DecodeGraphs":
        return DecodeGraphs(self, batch, prompt, new, groups)


def batch_view(cache, start: int, size: int):
    """The KV cache of sequences [start, start + size) of `cache`: views of its
    per-layer K / V tensors (the batch is the leading, outermost dimension)."""
    view = copy.copy(cache)
    view.k = [t[start:start + size] for t in cache.k]
    view.v = [t[start:start + size] for t in cache.v]
    view.batch = size
    return view


class DecodeGraphs:
    """One captured CUDA graph per decode step (positions are baked into the
    kernel arguments), replayed in capture order.  Owns the KV cache and the
    token buffer the graphs read and write.

    With `groups` > 1 the batch is split into that many equal groups of
    sequences; each group replays its own graphs on its own stream, with its
    own graph memory pool and scratch slot.  A decode step is a chain of
    latency-bound launches that leaves most SMs idle, so the groups' chains
    overlap on the GPU.  Every kernel computes a sequence's row with the same
    arithmetic whatever the batch, so the tokens are the same as with one
    group."""

    def __init__(self, model, batch: int, prompt: int, new: int, groups: int = 1):
        if groups < 1 or batch % groups:
            raise ValueError("groups must divide the batch")
        self.batch, self.prompt, self.new, self.groups = batch, prompt, new, groups
        self.cache = model.new_cache(batch, prompt + new)
        self.toks = torch.zeros((new, batch), dtype=torch.int64, device=model.device)
        bg = batch // groups
        self.views = [self.cache] if groups == 1 else [batch_view(self.cache, g * bg, bg) for g in range(groups)]
        self.streams = [None] if groups == 1 else [torch.cuda.Stream(device=model.device) for _ in range(groups)]
        c = model.cfg
        # the scratch buffer the last step's attention (or the LM-head argmax)
        # needs is reserved before any capture (graphs record its address), then one eager step
        # sets up per-kernel attributes and the small-M workspace
        need = max(ops.attention_workspace_bytes(bg, 1, c.n_head, c.n_kv_head, prompt + new - 1),
                   ops.linear_argmax_workspace_bytes(bg, c.vocab_size))
        self.graphs = []
        for g, (view, stream) in enumerate(zip(self.views, self.streams)):
            lo = g * bg
            with ops.workspace_slot(g):
                ops.reserve_workspace(model.device, need)
                view.length = prompt
                model.forward(self.toks[0, lo:lo + bg].view(bg, 1), view, last_only=True,
                              next_token=torch.empty_like(self.toks[0, lo:lo + bg]))
                torch.cuda.synchronize()
                pool = torch.cuda.graph_pool_handle()  # one pool per group: groups replay concurrently
                graphs = []
                for step in range(1, new):
                    view.length = prompt + step - 1
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, pool=pool, stream=stream):
                        model.forward(self.toks[step - 1, lo:lo + bg].view(bg, 1), view, last_only=True,
                                      next_token=self.toks[step, lo:lo + bg])
                    graphs.append(gr)
                self.graphs.append(graphs)
                view.length = 0
        self.cache.length = 0

    def replay(self):
        if self.groups == 1:
            for gr in self.graphs[0]:
                gr.replay()
        else:
            cur = torch.cuda.current_stream()
            for st in self.streams:
                st.wait_stream(cur)
            for step in range(self.new - 1):  # interleaved, so both groups start at once
                for graphs, st in zip(self.graphs, self.streams):
                    with torch.cuda.stream(st):
                        graphs[step].replay()
            for st in self.streams:
                cur.wait_stream(st)
        self.cache.length = self.prompt + self.new - 1
        for view in self.views:
            view.length = self.cache.length
