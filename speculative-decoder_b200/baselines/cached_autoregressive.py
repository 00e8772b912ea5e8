"""Plain cached decoding, the non-speculative baseline (interface of the reference's
baselines/cached_autoregressive.py:11-90).

Greedy decoding runs on the engine as one CUDA-graph replay per token
(specb200.plain.PlainDecoder): prefill, then per step the T = 1 forward, the device argmax
(first maximum, ties to the lowest id as torch.argmax) and the hand-off of the token to the
next step, with one small D2H of the tokens for eos and the output lists. It goes through the
same forward kernels as the speculative round, so speculative greedy output can be compared
with it token for token.

At temperature > 0 each token is drawn with torch.multinomial from the caller's generator on
the host, as lm/sampling.py:4-10 draws it, so seeded runs consume the generator exactly as the
reference does; that path runs one engine forward per step without a graph.
"""
from __future__ import annotations

from collections.abc import Callable

import torch
from transformers import PreTrainedModel

from cache.kv import KVCache
from lm.forward import forward
from lm.sampling import next_token
from specb200 import ops
from specb200.engine import engine_for
from specb200.plain import PlainDecoder


def _first_argmax(logits: torch.Tensor) -> torch.Tensor:
    """First maximum of each row of [B, V] logits, on the device (greedy fused sampler)."""
    b, v = logits.shape
    _, tok = ops.accept(logits.reshape(b, 1, v), None, None, None, torch.zeros(b, device=logits.device), logits=True,
                        temperature=0.0)
    return tok


def _decode(model: PreTrainedModel, cache: KVCache, seq_ids: list[int], prompts: list[list[int]], max_new_tokens: int,
            temperature: float, generator: torch.Generator | None, eos_id: int | None,
            on_event: Callable[[str], None] | None) -> list[list[int]]:
    """Decode every row until it emits eos or holds max_new_tokens; rows leave the batch (and
    free their cache) as they finish. The caller has added seq_ids to the cache."""
    width = max(len(p) for p in prompts)
    ids = torch.tensor([p + [0] * (width - len(p)) for p in prompts], dtype=torch.int64)
    logits = forward(model, cache, seq_ids, ids, [len(p) for p in prompts], last_only=True)
    outputs: list[list[int]] = [[] for _ in prompts]
    active = list(range(len(prompts)))
    dec = None
    if temperature == 0.0:
        first = _first_argmax(logits)
        tokens = first.tolist()
        dec = PlainDecoder(engine_for(model), cache, seq_ids, width + max_new_tokens + 1)
        dec.start(first)
    else:
        tokens = [next_token(row, temperature, generator) for row in logits]
    while True:
        for i in active:
            outputs[i].append(tokens[i] if dec is not None else tokens[active.index(i)])
        if on_event and all(len(o) == 1 for o in outputs):
            on_event("first_token")
        still = []
        for i in active:
            if outputs[i][-1] == eos_id or len(outputs[i]) == max_new_tokens:
                cache.free(seq_ids[i])
            else:
                still.append(i)
        active = still
        if not active:
            return outputs
        if dec is not None:
            tokens = dec.step(active)
        else:
            step_ids = torch.tensor([[outputs[i][-1]] for i in active])
            step_logits = forward(model, cache, [seq_ids[i] for i in active], step_ids, [1] * len(active))[:, 0]
            tokens = [next_token(row, temperature, generator) for row in step_logits]


@torch.no_grad()
def generate(model: PreTrainedModel, cache: KVCache, prompt: list[int], max_new_tokens: int,
             temperature: float = 0.0, generator: torch.Generator | None = None, eos_id: int | None = None,
             seq_id: int = 0, on_event: Callable[[str], None] | None = None) -> list[int]:
    """One prompt; returns its generated tokens (eos included when emitted)."""
    cache.add(seq_id)
    try:
        return _decode(model, cache, [seq_id], [prompt], max_new_tokens, temperature, generator, eos_id, on_event)[0]
    finally:
        if seq_id in cache.tables:
            cache.free(seq_id)


@torch.no_grad()
def generate_batch(model: PreTrainedModel, cache: KVCache, prompts: list[list[int]], max_new_tokens: int,
                   temperature: float = 0.0, generator: torch.Generator | None = None, eos_id: int | None = None,
                   on_event: Callable[[str], None] | None = None) -> list[list[int]]:
    """Several prompts decoded together, one step over every row still running; a row leaves
    when it emits eos or reaches max_new_tokens, as rows leave the speculative loop."""
    seq_ids = list(range(len(prompts)))
    for s in seq_ids:
        cache.add(s)
    try:
        return _decode(model, cache, seq_ids, prompts, max_new_tokens, temperature, generator, eos_id, on_event)
    finally:
        for s in seq_ids:
            if s in cache.tables:
                cache.free(s)
