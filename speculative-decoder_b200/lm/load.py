"""Model construction helpers (lm/load.py of the reference).

`tiny_model` keeps the reference's seed-then-construct recipe (lm/load.py:124-141), so a
seed gives the same weights on both sides of a parity test. `load_model` wraps
from_pretrained at a pinned revision; the engine packs the weights itself on first use
(specb200.engine), so `pack` only moves the model to its device.
"""
from __future__ import annotations

from typing import Any

import torch
from transformers import (
    AutoConfig,
    AutoModelForCausalLM,
    AutoTokenizer,
    LlamaConfig,
    LlamaForCausalLM,
    PretrainedConfig,
    PreTrainedModel,
    PreTrainedTokenizerBase,
)

from lm.forward import check_supported


class VocabMismatch(ValueError):
    pass


def resolve_device(name: str) -> torch.device:
    if name != "auto":
        return torch.device(name)
    return torch.device("cuda" if torch.cuda.is_available() else "cpu")


def load_model(spec: dict[str, Any], cache_dir: str, device: torch.device, dtype: str | None = None,
               local_files_only: bool = False) -> PreTrainedModel:
    model = AutoModelForCausalLM.from_pretrained(
        spec["repo"], revision=spec["revision"], cache_dir=cache_dir, local_files_only=local_files_only,
        dtype=getattr(torch, dtype or spec["dtype"]), attn_implementation="sdpa")
    pack(model, device)
    model.eval()
    check_supported(model)
    return model


def pack(model: PreTrainedModel, device: torch.device) -> None:
    model.to(device)


def load_config(spec: dict[str, Any], cache_dir: str) -> PretrainedConfig:
    return AutoConfig.from_pretrained(spec["repo"], revision=spec["revision"], cache_dir=cache_dir)


def load_tokenizer(spec: dict[str, Any], cache_dir: str, local_files_only: bool = False) -> PreTrainedTokenizerBase:
    return AutoTokenizer.from_pretrained(spec["repo"], revision=spec["revision"], cache_dir=cache_dir,
                                         local_files_only=local_files_only)


def check_shared_vocab(target: PretrainedConfig, draft: PretrainedConfig, target_tok: PreTrainedTokenizerBase,
                       draft_tok: PreTrainedTokenizerBase) -> None:
    """Accept-reject compares p(x) and q(x) id by id, so both models must mean the same
    string by every id (lm/load.py:107-121)."""
    if target.vocab_size != draft.vocab_size:
        raise VocabMismatch(f"logit width: target {target.vocab_size}, draft {draft.vocab_size}")
    if target_tok.get_vocab() != draft_tok.get_vocab():
        raise VocabMismatch("tokenizer vocabularies differ")
    if target_tok.eos_token_id != draft_tok.eos_token_id:
        raise VocabMismatch(f"eos id: target {target_tok.eos_token_id}, draft {draft_tok.eos_token_id}")


def tiny_model(seed: int, vocab_size: int = 256, n_layers: int = 2, hidden: int = 64,
               dtype: torch.dtype = torch.float32) -> LlamaForCausalLM:
    """2-layer Llama with 4 query heads over 2 KV heads (grouped-query attention exercised)."""
    config = LlamaConfig(vocab_size=vocab_size, hidden_size=hidden, intermediate_size=2 * hidden,
                         num_hidden_layers=n_layers, num_attention_heads=4, num_key_value_heads=2,
                         max_position_embeddings=1024, attn_implementation="sdpa")
    torch.manual_seed(seed)
    model = LlamaForCausalLM(config).to(dtype).eval()
    check_supported(model)
    return model
