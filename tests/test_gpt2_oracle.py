"""The GPT-2 oracle against Hugging Face transformers (CPU only).

The reference validates its GPT-2 forward against the HF model's logits
(examples/gpt2/gpt2_inference.py, README "validates output against the
HuggingFace reference").  The same comparison pins the oracle here: HF
`GPT2LMHeadModel` in fp32 and the oracle (which rounds to bf16 where the
reference's GPU kernels do) run on identical seeded random weights; no
network or pretrained checkpoint is needed.
"""

import pytest
import torch

from oracle.gpt2 import OracleGPT2
from xb200.gpt2 import GPT2Config, random_weights

transformers = pytest.importorskip("transformers")

TINY = GPT2Config(n_layer=2, n_head=4, n_embd=256, vocab_size=1000, n_positions=128)


def _hf(cfg, sd):
    from transformers import GPT2Config as HFConfig, GPT2LMHeadModel

    hc = HFConfig(vocab_size=cfg.vocab_size, n_positions=cfg.n_positions, n_embd=cfg.n_embd, n_layer=cfg.n_layer,
                  n_head=cfg.n_head, layer_norm_epsilon=cfg.ln_eps, activation_function="gelu_new",
                  resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0, tie_word_embeddings=True)
    model = GPT2LMHeadModel(hc).eval().float()
    fsd = {k: v.float() for k, v in sd.items()}
    fsd["lm_head.weight"] = fsd["transformer.wte.weight"]
    missing, unexpected = model.load_state_dict(fsd, strict=False)
    assert not [m for m in missing if not m.endswith("attn.bias") and "masked_bias" not in m], missing
    return model


def _metrics(a, b):
    a, b = a.reshape(-1, a.shape[-1]).double(), b.reshape(-1, b.shape[-1]).double()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=-1)
    top1 = (a.argmax(-1) == b.argmax(-1)).double().mean()
    return float(cos.min()), float(top1), float((a - b).abs().max()), float(b.abs().max())


@pytest.mark.parametrize("cfg,std", [(TINY, 0.05), (GPT2Config.variant("gpt2"), 0.02)])
def test_oracle_prefill_matches_hf(cfg, std):
    sd = random_weights(cfg, seed=3, std=std)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (2, 24), generator=g)
    orc = OracleGPT2(sd, cfg)
    got = orc.forward(ids, orc.new_cache(2, 24))
    with torch.no_grad():
        ref = _hf(cfg, sd)(ids).logits
    cos_min, top1, maxdiff, scale = _metrics(got, ref)
    assert cos_min > 0.999, cos_min
    assert top1 > 0.9, top1
    assert maxdiff < 0.05 * scale + 1e-2, (maxdiff, scale)


def test_oracle_kv_cache_decode_matches_hf_full_sequence():
    sd = random_weights(TINY, seed=4, std=0.05)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, TINY.vocab_size, (1, 20), generator=g)
    orc = OracleGPT2(sd, TINY)
    cache = orc.new_cache(1, 20)
    orc.forward(ids[:, :16], cache)
    steps = [orc.forward(ids[:, t:t + 1], cache)[:, -1] for t in range(16, 20)]
    with torch.no_grad():
        full = _hf(TINY, sd)(ids).logits[:, 16:20]
    got = torch.stack(steps, 1)
    cos_min, top1, maxdiff, scale = _metrics(got, full)
    assert cos_min > 0.999 and top1 == 1.0, (cos_min, top1)


def test_variant_table():
    assert [(GPT2Config.variant(n).n_layer, GPT2Config.variant(n).head_dim) for n in
            ("gpt2", "gpt2-medium", "gpt2-large", "gpt2-xl")] == [(12, 64), (24, 64), (36, 64), (48, 64)]
