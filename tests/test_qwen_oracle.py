"""The Qwen2.5 oracle against Hugging Face transformers (CPU only).

The reference checks its Qwen forward against the HF model with logit
metrics -- max / mean abs difference, cosine similarity, top-1 / top-5
agreement (examples/qwen2_5/qwen_inference.py:92-129).  The same comparison
pins the oracle here: HF `Qwen2ForCausalLM` in fp32 and the oracle (which
rounds to bf16 where the reference's GPU kernels do) run on identical
seeded random weights; no network or pretrained checkpoint is needed.
"""

import pytest
import torch

from oracle.qwen import OracleQwen
from xb200.qwen import QwenConfig, random_weights

transformers = pytest.importorskip("transformers")

TINY = QwenConfig(n_layer=2, n_head=4, n_kv_head=2, n_embd=256, head_dim=64, intermediate=512, vocab_size=1024,
                  max_seq_len=4096)


def _hf(cfg, sd):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    hc = Qwen2Config(vocab_size=cfg.vocab_size, hidden_size=cfg.n_embd, intermediate_size=cfg.intermediate,
                     num_hidden_layers=cfg.n_layer, num_attention_heads=cfg.n_head,
                     num_key_value_heads=cfg.n_kv_head, max_position_embeddings=cfg.max_seq_len,
                     rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_eps, tie_word_embeddings=True,
                     torch_dtype=torch.float32)
    model = Qwen2ForCausalLM(hc).eval()
    fsd = {k: v.float() for k, v in sd.items()}
    fsd["lm_head.weight"] = fsd["model.embed_tokens.weight"]
    missing, unexpected = model.load_state_dict(fsd, strict=False)
    assert not [m for m in missing if "rotary" not in m], missing
    return model


def _metrics(a, b):
    a, b = a.reshape(-1, a.shape[-1]).double(), b.reshape(-1, b.shape[-1]).double()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=-1)
    top1 = (a.argmax(-1) == b.argmax(-1)).double().mean()
    return float(cos.min()), float(top1), float((a - b).abs().max()), float(b.abs().max())


def test_oracle_prefill_matches_hf():
    sd = random_weights(TINY, seed=3, std=0.05)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, TINY.vocab_size, (2, 24), generator=g)
    orc = OracleQwen(sd, TINY)
    got = orc.forward(ids, orc.new_cache(2, 24))
    with torch.no_grad():
        ref = _hf(TINY, sd)(ids).logits
    cos_min, top1, maxdiff, scale = _metrics(got, ref)
    assert cos_min > 0.999, cos_min
    assert top1 > 0.9, top1
    assert maxdiff < 0.05 * scale + 1e-2, (maxdiff, scale)


def test_oracle_kv_cache_decode_matches_hf_full_sequence():
    sd = random_weights(TINY, seed=4, std=0.05)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, TINY.vocab_size, (1, 20), generator=g)
    orc = OracleQwen(sd, TINY)
    cache = orc.new_cache(1, 20)
    orc.forward(ids[:, :16], cache)
    steps = [orc.forward(ids[:, t:t + 1], cache)[:, -1] for t in range(16, 20)]
    with torch.no_grad():
        full = _hf(TINY, sd)(ids).logits[:, 16:20]
    got = torch.stack(steps, 1)
    cos_min, top1, maxdiff, scale = _metrics(got, full)
    assert cos_min > 0.999 and top1 == 1.0, (cos_min, top1)


def test_oracle_gqa_matches_repeat_interleave():
    # the oracle's attention is exactly the reference's expand-then-attend
    from oracle.qwen import attention

    g = torch.Generator().manual_seed(2)
    q = torch.randn(1, 4, 5, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(1, 2, 5, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(1, 2, 5, 64, generator=g).to(torch.bfloat16)
    out = attention(q, k, v, 0, 0.125)
    for h in range(4):
        s = (q[0, h].float() @ k[0, h // 2].float().t()) * 0.125
        s = s.masked_fill(torch.triu(torch.ones(5, 5, dtype=torch.bool), 1), float("-inf"))
        p = torch.softmax(s, -1)
        ref = (p @ v[0, h // 2].float()).to(torch.bfloat16)
        torch.testing.assert_close(out[0, h].float(), ref.float(), atol=2e-2, rtol=2e-2)
