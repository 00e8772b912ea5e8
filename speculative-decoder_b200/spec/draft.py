"""Drafters for the speculative round, on the B200 engine.

The `Drafter` protocol is the reference's (spec/draft.py:12-24): a drafter proposes k tokens
per row together with the distributions q it drew them from, and keeps whatever state it has
(a KV cache) in step with the round through prefill / rollback / release.

`ModelDraft` proposes with a small language model. Where the reference runs k Python-level
forward calls and copies each step's probabilities to the host (spec/draft.py:42-56), the
engine runs the k steps as one device-resident launch sequence (specb200.draftloop.DraftSteps:
forward, fused sampler and token scatter per step) and returns the drafts and q on the GPU;
only the draft cache's block bookkeeping and the uniforms are prepared on the host. The
round driver's CUDA-graph path (specb200.rounds) replays the same launch sequence inside its
round graph.

`NoisyDraft` is the noisy-copy drafter of BASELINE config 2's second variant, which the
reference does not have: the target model itself, with seeded N(0, sigma^2) noise added to its
final logits (sigma sets the acceptance rate).

`UniformDraft` is the reference's worst-case drafter (spec/draft.py:64-85), kept for the
exactness tests, and `run` is its right-padded last-token forward (spec/draft.py:88-92).
"""
from __future__ import annotations

from typing import Protocol

import torch
from transformers import PreTrainedModel

from cache.kv import KVCache
from lm.forward import forward
from specb200 import _ffi, ops
from specb200.draftloop import DraftSteps
from specb200.engine import engine_for


class Drafter(Protocol):
    def prefill(self, seq_ids: list[int], prompts: list[list[int]]) -> None: ...

    def propose(self, seq_ids: list[int], contexts: list[list[int]], k: int, temperature: float,
                generator: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
        """k proposed tokens per row, [B, k], and the distributions they were drawn from,
        [B, k, V]. Accept-reject is exact only if q is what the tokens were sampled from."""
        ...

    def rollback(self, seq_id: int, keep: int) -> None: ...

    def release(self, seq_id: int) -> None: ...


def _uniforms(n: int, generator: torch.Generator | None, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """One uniform per row, drawn where the generator lives (the reference's draw in
    spec/draft.py:27-29, one call per sampled step)."""
    where = generator.device if generator is not None else torch.device("cpu")
    return torch.rand(n, generator=generator, dtype=dtype, device=where)


def sample(probs: torch.Tensor, generator: torch.Generator) -> torch.Tensor:
    """Inverse-CDF sample of each row of probs [B, V] under one uniform per row from the
    caller's generator (spec/draft.py:27-29), on the fused kernel."""
    from spec.accept import sample_inverse_cdf

    return sample_inverse_cdf(probs, _uniforms(probs.shape[0], generator, probs.dtype))


def run(model: PreTrainedModel, cache: KVCache, seq_ids: list[int], chunks: list[list[int]]) -> torch.Tensor:
    """Append each row's chunk to its sequence and return the logits after the chunk's last
    token, [B, V] (rows right-padded to the longest chunk)."""
    lengths = [len(c) for c in chunks]
    width = max(lengths)
    padded = torch.tensor([c + [0] * (width - len(c)) for c in chunks], dtype=torch.int64)
    return forward(model, cache, seq_ids, padded, lengths, last_only=True)


class ModelDraft:
    """A draft language model with its own paged KV cache. The cache trails the context by
    one token (the round's last emitted token is fed at the next proposal), or by two after a
    round that accepted all k drafts (the last draft token was sampled but never fed)."""

    _CAP_STEP = 256  # contexts are planned in multiples of this many positions

    def __init__(self, model: PreTrainedModel, cache: KVCache) -> None:
        self.model = model
        self.cache = cache
        self._steps: dict[tuple[int, int, float, int], DraftSteps] = {}

    def prefill(self, seq_ids: list[int], prompts: list[list[int]]) -> None:
        for s in seq_ids:
            self.cache.add(s)
        run(self.model, self.cache, seq_ids, prompts)

    def noise(self) -> tuple[float, int] | None:
        """(sigma, seed) of the logit noise this drafter adds, or None."""
        return None

    def _steps_for(self, rows: int, k: int, temperature: float, longest: int) -> DraftSteps:
        cap = -(-(longest + k + 2) // self._CAP_STEP) * self._CAP_STEP
        key = (rows, k, float(temperature), cap)
        if key not in self._steps:
            self._steps[key] = DraftSteps(engine_for(self.model), self.cache, rows, k, cap, temperature,
                                          noise=self.noise())
        return self._steps[key]

    def propose(self, seq_ids: list[int], contexts: list[list[int]], k: int, temperature: float,
                generator: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
        rows = len(seq_ids)
        steps = self._steps_for(rows, k, temperature, max(len(c) for c in contexts))
        # host side, in the reference's order: the cache grows by the pending tokens, then by
        # one position per later step; each step consumes one uniform per row
        past, grow, pending = steps.plan(seq_ids, contexts)
        u = torch.stack([_uniforms(rows, generator) for _ in range(k)])
        ids0 = torch.zeros(rows, 2, dtype=torch.int32)
        for i, p in enumerate(pending):
            ids0[i, : len(p)] = torch.tensor(p, dtype=torch.int32)
        table = torch.zeros_like(steps.table, device="cpu")
        for i, s in enumerate(seq_ids):
            blocks = self.cache.tables[s].blocks
            table[i, : len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
        steps.ids0.copy_(ids0)
        steps.past.copy_(torch.tensor(past, dtype=torch.int32))
        steps.n_new.copy_(torch.tensor(grow, dtype=torch.int32))
        steps.table.copy_(table)
        steps.u.copy_(u)
        steps.row_ids.copy_(torch.tensor(seq_ids, dtype=torch.int32))
        # device side: k x (forward, sampler, scatter), nothing comes back in between
        steps.launch()
        _ffi.check_status(steps.status, "draft steps")
        q = ops.probabilities(steps.q_logits, temperature).transpose(0, 1).contiguous()
        return steps.draft.clone(), q

    def rollback(self, seq_id: int, keep: int) -> None:
        # the cache may hold fewer than `keep` positions (it trails the context)
        self.cache.truncate(seq_id, min(keep, self.cache.length(seq_id)))

    def release(self, seq_id: int) -> None:
        self.cache.free(seq_id)


class NoisyDraft(ModelDraft):
    """Drafts with the target itself, adding sigma * z to each step's final logits before they
    become q (BASELINE config 2's second variant; the reference has no such drafter). z is a
    standard normal per (seed, sequence id, position of the predicted token, vocabulary id)
    from Philox4x32-10 (specb200_logit_noise), so the oracle reproduces it; the q handed to
    accept-reject is the softmax of the noisy logits, the distribution the drafts were drawn
    from. Pass the target model and a KV cache of its own."""

    def __init__(self, model: PreTrainedModel, cache: KVCache, sigma: float, seed: int = 0) -> None:
        super().__init__(model, cache)
        if not sigma >= 0:
            raise ValueError(f"sigma must be >= 0, got {sigma}")
        self.sigma, self.seed = float(sigma), int(seed)

    def noise(self) -> tuple[float, int] | None:
        return self.sigma, self.seed


class UniformDraft:
    """Proposes uniformly random tokens with q = 1/V everywhere: acceptance near 1/V, and the
    output must still be exactly the target's."""

    def __init__(self, vocab_size: int) -> None:
        self.vocab_size = vocab_size

    def prefill(self, seq_ids: list[int], prompts: list[list[int]]) -> None:
        return None

    def propose(self, seq_ids: list[int], contexts: list[list[int]], k: int, temperature: float,
                generator: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
        tokens = torch.randint(0, self.vocab_size, (len(seq_ids), k), generator=generator)
        dev = torch.device("cuda", torch.cuda.current_device())
        return tokens, torch.full((len(seq_ids), k, self.vocab_size), 1.0 / self.vocab_size, device=dev)

    def rollback(self, seq_id: int, keep: int) -> None:
        return None

    def release(self, seq_id: int) -> None:
        return None
