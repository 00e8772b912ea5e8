"""Seeded model and prompt recipes for the BASELINE configurations, shared by the golden-vector
script (which runs the reference on them) and the GPU tests (which run the engine on them).

Only torch and transformers are used, so the same weights come out in any process that runs
the same torch build: the reference's tests build their models the same way
(lm/load.py:124-141: a LlamaConfig, torch.manual_seed, LlamaForCausalLM, HF's N(0, 0.02) init
with RMSNorm weights at 1).
"""
from __future__ import annotations

import torch

# SmolLM2-135M architecture (BASELINE configs 1 and 2's draft)
SMOL_135M = dict(hidden_size=576, num_hidden_layers=30, num_attention_heads=9, num_key_value_heads=3,
                 intermediate_size=1536, vocab_size=49152, rope_theta=100000.0)
# SmolLM2-1.7B architecture (4 and 5's target)
SMOL_1P7B = dict(hidden_size=2048, num_hidden_layers=24, num_attention_heads=32, num_key_value_heads=32,
                 intermediate_size=8192, vocab_size=49152, rope_theta=130000.0)


def llama(spec: dict, seed: int, dtype: torch.dtype = torch.float32, layers: int | None = None):
    """Random-init Llama of the given architecture: weights drawn in fp32 under
    torch.manual_seed(seed), then cast to `dtype`."""
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=spec["vocab_size"], hidden_size=spec["hidden_size"],
                      intermediate_size=spec["intermediate_size"],
                      num_hidden_layers=layers or spec["num_hidden_layers"],
                      num_attention_heads=spec["num_attention_heads"],
                      num_key_value_heads=spec["num_key_value_heads"], max_position_embeddings=8192,
                      rms_norm_eps=1e-5, rope_parameters={"rope_type": "default", "rope_theta": spec["rope_theta"]},
                      tie_word_embeddings=True, initializer_range=0.02, attn_implementation="sdpa")
    torch.manual_seed(seed)
    model = LlamaForCausalLM(cfg)
    return model.to(dtype).eval()


def config1_prompt(seed: int = 0) -> list[int]:
    """BASELINE config 1's prompt: a 32-id uniform-random segment repeated 8 times (256 ids)."""
    seg = torch.randint(0, SMOL_135M["vocab_size"], (32,), generator=torch.Generator().manual_seed(seed)).tolist()
    return seg * 8


def uniform_prompt(n: int, vocab: int, seed: int) -> list[int]:
    """n uniform-random ids (BASELINE configs 2 and 4)."""
    return torch.randint(0, vocab, (n,), generator=torch.Generator().manual_seed(seed)).tolist()


def segment_prompt(n: int, vocab: int, seed: int, seg: int = 64, p_repeat: float = 0.5) -> list[int]:
    """BASELINE config 5's prompt: 64-id uniform-random segments, each followed by a copy of
    itself with probability 0.5, cut to n ids."""
    g = torch.Generator().manual_seed(seed)
    out: list[int] = []
    while len(out) < n:
        s = torch.randint(0, vocab, (seg,), generator=g).tolist()
        out += s
        if float(torch.rand(1, generator=g)) < p_repeat:
            out += s
    return out[:n]
