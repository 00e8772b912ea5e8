"""The speculative round driver (reference spec/loop.py:14-129) on the B200 engine.

`generate` keeps the reference's signature, events, statistics and per-row bookkeeping:
the first token comes from the target's prefill logits, then each round proposes k tokens,
verifies them in one (k+1)-token target forward, accepts a prefix plus one corrected or
bonus token, trims at the budget/eos, and rolls the target cache back to
len(context) - 1 + (accepted) with a table edit. The generator is consumed in the
reference's order, so seeded runs draw the same uniforms.

Two execution paths share these semantics:
  * the fused path (specb200.rounds), taken when the drafter is one of the engine's own
    (NGramDraft, ModelDraft) and `verify` / `accept_reject` are this module's: contexts,
    drafts and uniforms live on the device, the round (draft kernels, verify forward,
    fused logits->accept kernel, context commit) is replayed from a CUDA graph, and the host
    reads back 3 small integers per row per round;
  * the composable path below for any other drafter, or when a caller has replaced
    `spec.loop.verify` / `spec.loop.accept_reject` (the reference's tests do): the same
    kernels, called one module function at a time.
"""
from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, field

import torch
from transformers import PreTrainedModel

from cache.kv import KVCache
from lm.sampling import probabilities
from spec.accept import accept_reject
from spec.draft import Drafter, run, sample
from spec.verify import verify


@dataclass
class SpecStats:
    k: int
    rounds: int = 0
    drafted: int = 0
    accepted: int = 0
    # attempts[i]: rounds that reached draft position i; accepts[i]: of those, accepted there.
    attempts: list[int] = field(default_factory=list)
    accepts: list[int] = field(default_factory=list)
    # One entry per (sequence, round): tokens emitted that round, after eos/budget trimming.
    emitted_per_round: list[int] = field(default_factory=list)
    # Same indexing: how many of the emitted tokens were accepted draft tokens.
    drafted_per_round: list[int] = field(default_factory=list)

    def __post_init__(self) -> None:
        self.attempts = [0] * self.k
        self.accepts = [0] * self.k

    @property
    def discarded(self) -> int:
        return self.drafted - self.accepted


def record(stats: SpecStats, n: int) -> None:
    stats.drafted += stats.k
    stats.accepted += n
    for i in range(min(n + 1, stats.k)):
        stats.attempts[i] += 1
    for i in range(n):
        stats.accepts[i] += 1


def trim(new: list[int], have: int, max_new_tokens: int, eos_id: int | None) -> list[int]:
    new = new[: max_new_tokens - have]
    if eos_id is not None and eos_id in new:
        new = new[: new.index(eos_id) + 1]
    return new


def finished(output: list[int], max_new_tokens: int, eos_id: int | None) -> bool:
    return len(output) >= max_new_tokens or (eos_id is not None and output[-1] == eos_id)


def release(cache: KVCache, drafter: Drafter, seq_id: int) -> None:
    cache.free(seq_id)
    drafter.release(seq_id)


def settle_row(stats: SpecStats, cache: KVCache, drafter: Drafter, s: int, n: int, draft_row: list[int],
               next_token: int, contexts: list[list[int]], outputs: list[list[int]], max_new_tokens: int,
               eos_id: int | None) -> bool:
    """Book one row's round result; returns True while the row stays active. The target
    cache holds context[:-1] plus the k+1 verified positions; after keeping n drafts and
    one corrected/bonus token the context has L + n + 1 tokens and the cache must hold
    L + n of them, so entries for d_{n+1}..d_k are dropped (reference spec/loop.py:92-99)."""
    record(stats, n)
    new = trim(draft_row[:n] + [next_token], len(outputs[s]), max_new_tokens, eos_id)
    stats.emitted_per_round.append(len(new))
    stats.drafted_per_round.append(min(n, len(new)))
    length_before = len(contexts[s])
    contexts[s] = contexts[s] + new
    outputs[s] = outputs[s] + new
    if finished(outputs[s], max_new_tokens, eos_id):
        release(cache, drafter, s)
        return False
    cache.truncate(s, length_before + n)
    drafter.rollback(s, length_before + n)
    return True


@torch.no_grad()
def generate(
    target: PreTrainedModel,
    cache: KVCache,
    drafter: Drafter,
    prompts: list[list[int]],
    max_new_tokens: int,
    k: int,
    temperature: float = 0.0,
    generator: torch.Generator | None = None,
    eos_id: int | None = None,
    on_event: Callable[[str], None] | None = None,
) -> tuple[list[list[int]], SpecStats]:
    generator = generator or torch.Generator().manual_seed(0)
    on_event = on_event or (lambda name: None)
    from specb200 import rounds

    if rounds.fused_path_available(drafter, verify, accept_reject):
        return rounds.generate_fused(target, cache, drafter, prompts, max_new_tokens, k, temperature, generator,
                                     eos_id, on_event)

    stats = SpecStats(k)
    seq_ids = list(range(len(prompts)))
    for seq_id in seq_ids:
        cache.add(seq_id)
    # The first token comes from the target's prefill logits, as in plain decoding, and is
    # emitted before the draft does any work.
    first = sample(probabilities(run(target, cache, seq_ids, prompts), temperature), generator).tolist()
    on_event("first_token")
    drafter.prefill(seq_ids, prompts)
    on_event("draft_prefilled")
    contexts = [p + [t] for p, t in zip(prompts, first)]
    outputs = [[t] for t in first]
    active = [s for s in seq_ids if not finished(outputs[s], max_new_tokens, eos_id)]
    for s in seq_ids:
        if s not in active:
            release(cache, drafter, s)

    while active:
        ctx = [contexts[s] for s in active]
        draft, q = drafter.propose(active, ctx, k, temperature, generator)
        p = verify(target, cache, active, ctx, draft, temperature)
        verdict = accept_reject(p, q, draft, generator=generator)
        stats.rounds += 1
        n_acc = verdict.n_accepted.tolist()
        nxt = verdict.next_token.tolist()
        drafts = draft.tolist()
        active = [s for row, s in enumerate(active)
                  if settle_row(stats, cache, drafter, s, int(n_acc[row]), drafts[row], int(nxt[row]), contexts,
                                outputs, max_new_tokens, eos_id)]
        if stats.rounds == 1:
            on_event("first_round")
    return outputs, stats
