"""Drafters (reference spec/draft.py:12-92) on the B200 engine.

`ModelDraft` runs the draft model's forward through the same kernels as the target; its
q rows stay on the device. `run` is the reference's right-padded last-token forward and
`sample` the inverse-CDF sampler, with the uniform drawn from the caller's generator as the
reference draws it (spec/draft.py:27-29).
"""
from __future__ import annotations

from typing import Protocol

import torch
from transformers import PreTrainedModel

from cache.kv import KVCache
from lm.forward import forward
from lm.sampling import probabilities
from spec.accept import sample_inverse_cdf


class Drafter(Protocol):
    def prefill(self, seq_ids: list[int], prompts: list[list[int]]) -> None: ...

    def propose(self, seq_ids: list[int], contexts: list[list[int]], k: int, temperature: float,
                generator: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
        """Returns draft [B, k] and q [B, k, V]: the distributions the draft tokens were
        actually sampled from. Accept-reject is exact only against those."""
        ...

    def rollback(self, seq_id: int, keep: int) -> None: ...

    def release(self, seq_id: int) -> None: ...


def sample(probs: torch.Tensor, generator: torch.Generator) -> torch.Tensor:
    where = generator.device if generator is not None else torch.device("cpu")
    u = torch.rand(probs.shape[0], generator=generator, dtype=probs.dtype, device=where)
    return sample_inverse_cdf(probs, u)


class ModelDraft:
    def __init__(self, model: PreTrainedModel, cache: KVCache) -> None:
        self.model = model
        self.cache = cache

    def prefill(self, seq_ids: list[int], prompts: list[list[int]]) -> None:
        for seq_id in seq_ids:
            self.cache.add(seq_id)
        run(self.model, self.cache, seq_ids, prompts)

    def propose(self, seq_ids: list[int], contexts: list[list[int]], k: int, temperature: float,
                generator: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
        # The draft cache lags the context by one token, or by two after a round in which
        # every draft was accepted (d_k was sampled but never fed); the first step feeds
        # every uncached token, which closes either gap.
        pending = [ctx[self.cache.length(s):] for s, ctx in zip(seq_ids, contexts)]
        tokens, qs = [], []
        for _ in range(k):
            q = probabilities(run(self.model, self.cache, seq_ids, pending), temperature)
            token = sample(q, generator)
            tokens.append(token)
            qs.append(q)
            pending = [[t] for t in token.tolist()]
        return torch.stack(tokens, dim=1), torch.stack(qs, dim=1)

    def rollback(self, seq_id: int, keep: int) -> None:
        self.cache.truncate(seq_id, min(self.cache.length(seq_id), keep))

    def release(self, seq_id: int) -> None:
        self.cache.free(seq_id)


class UniformDraft:
    """The worst useful draft: acceptance near 1/V, output must still be exact."""

    def __init__(self, vocab_size: int) -> None:
        self.vocab_size = vocab_size

    def prefill(self, seq_ids: list[int], prompts: list[list[int]]) -> None:
        pass

    def propose(self, seq_ids: list[int], contexts: list[list[int]], k: int, temperature: float,
                generator: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
        q = torch.full((len(seq_ids), k, self.vocab_size), 1.0 / self.vocab_size)
        return torch.randint(0, self.vocab_size, (len(seq_ids), k), generator=generator), q

    def rollback(self, seq_id: int, keep: int) -> None:
        pass

    def release(self, seq_id: int) -> None:
        pass


def run(model: PreTrainedModel, cache: KVCache, seq_ids: list[int], chunks: list[list[int]]) -> torch.Tensor:
    """Forward right-padded chunks; returns the logits after each row's last real token, [B, V]."""
    n_new = [len(c) for c in chunks]
    width = max(n_new)
    input_ids = torch.tensor([c + [0] * (width - len(c)) for c in chunks], dtype=torch.int64)
    return forward(model, cache, seq_ids, input_ids, n_new, last_only=True)
