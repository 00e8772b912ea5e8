"""Cached forward pass (lm/forward.py:21-84 of the reference) on the B200 engine.

`forward` keeps the reference's signature and meaning: run right-padded input_ids [B, T]
through the model, appending to each sequence's paged cache, and return fp32 logits
[B, T, V] (or each row's last real token, [B, V]). The work is one call into
libspecb200.so (embed, per-layer RMSNorm / QKV+RoPE+KV-write / paged attention / O /
gate-up+SiLU / down, final norm, fp32-accumulated head); nothing runs on the CPU.
"""
from __future__ import annotations

import torch
from transformers import PreTrainedModel

from cache.kv import KVCache
from specb200 import ops
from specb200.engine import engine_for

SUPPORTED = {"llama", "qwen2"}


def check_supported(model: PreTrainedModel) -> None:
    config = model.config
    if config.model_type not in SUPPORTED:
        raise NotImplementedError(f"cached forward supports {sorted(SUPPORTED)}, got {config.model_type}")
    if getattr(config, "use_sliding_window", False):
        raise NotImplementedError("sliding-window attention is not implemented")


@torch.no_grad()
def forward(model: PreTrainedModel, cache: KVCache, seq_ids: list[int], input_ids: torch.Tensor, n_new: list[int],
            last_only: bool = False) -> torch.Tensor:
    """Rows past n_new[b] are padding and their logits meaningless; padded tokens write no
    K/V. The same call serves prefill (T = prompt), decode (T = 1) and verify (T = k + 1)."""
    return engine_for(model).forward(cache, seq_ids, input_ids, n_new, last_only)


def logits(model: PreTrainedModel, hidden: torch.Tensor) -> torch.Tensor:
    """The output projection with fp32 accumulation (lm/forward.py:71-84). Every product of two
    bf16 values is exact in fp32, so the bf16 weight is streamed once and accumulated in fp32
    on the tensor cores instead of keeping an fp32 copy of it."""
    eng = engine_for(model)
    x = hidden.to(eng.device, eng.dtype)
    flat = x.reshape(-1, x.shape[-1])
    out = ops.linear(flat, eng.lm_head, out_f32=True)
    return out.reshape(*x.shape[:-1], eng.vocab)
