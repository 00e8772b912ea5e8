"""Oracle: the speculative round driver and plain cached decoding, in numpy.

Restates spec/loop.py:38-129 (generate: first token from prefill logits, propose -> verify
-> accept -> trim -> truncate/rollback, SpecStats bookkeeping), spec/draft.py:27-92
(sample, ModelDraft with its lag-closing first step, run), spec/ngram.py:4-29 (NGramDraft)
and baselines/cached_autoregressive.py:11-39 (plain greedy decoding) of the reference, on
top of oracle.forward and oracle.accept. Uniforms come from a torch CPU generator in the
reference's order, so a seeded oracle run consumes the same random stream.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import accept as acc
from oracle import forward as fw
from oracle import noise
from oracle.ngram import lookup_batch


def _rand(shape, generator: torch.Generator) -> np.ndarray:
    return torch.rand(*shape, generator=generator, dtype=torch.float32).numpy()


def sample(probs: np.ndarray, generator: torch.Generator) -> np.ndarray:
    """spec/draft.py:27-29."""
    return acc.sample_inverse_cdf(probs.astype(np.float32), _rand((probs.shape[0],), generator))


def run(w: dict, cache: fw.Cache, seq_ids: list[int], chunks: list[list[int]], prec: fw.Precision) -> np.ndarray:
    """spec/draft.py:87-92: right-padded chunks, logits after each row's last real token."""
    n_new = [len(c) for c in chunks]
    width = max(n_new)
    ids = np.array([c + [0] * (width - len(c)) for c in chunks], dtype=np.int64)
    return fw.forward(w, cache, seq_ids, ids, n_new, prec, last_only=True)


class NGramDraft:
    """spec/ngram.py:4-29."""

    def __init__(self, vocab_size: int, max_n: int = 3) -> None:
        self.vocab_size, self.max_n = vocab_size, max_n

    def prefill(self, seq_ids, prompts) -> None:
        pass

    def propose(self, seq_ids, contexts, k, temperature, generator):
        draft = lookup_batch(contexts, k, self.max_n)
        q = np.zeros((len(contexts), k, self.vocab_size), dtype=np.float32)
        np.put_along_axis(q, draft[..., None], 1.0, axis=-1)
        return draft, q

    def rollback(self, seq_id, keep) -> None:
        pass

    def release(self, seq_id) -> None:
        pass


class ModelDraft:
    """spec/draft.py:32-62."""

    def __init__(self, w: dict, prec: fw.Precision, num_blocks: int, block_size: int) -> None:
        self.w, self.prec = w, prec
        self.cache = fw.Cache(w, num_blocks, block_size, prec)

    def prefill(self, seq_ids, prompts) -> None:
        for s in seq_ids:
            self.cache.add(s)
        run(self.w, self.cache, seq_ids, prompts, self.prec)

    def _logits(self, seq_ids, pending) -> np.ndarray:
        return run(self.w, self.cache, seq_ids, pending, self.prec).astype(np.float32)

    def propose(self, seq_ids, contexts, k, temperature, generator):
        pending = [ctx[self.cache.length(s):] for s, ctx in zip(seq_ids, contexts)]
        tokens, qs = [], []
        for _ in range(k):
            q = acc.probabilities(self._logits(seq_ids, pending), temperature)
            tok = sample(q, generator)
            tokens.append(tok)
            qs.append(q)
            pending = [[int(t)] for t in tok]
        return np.stack(tokens, axis=1), np.stack(qs, axis=1)

    def rollback(self, seq_id, keep) -> None:
        self.cache.truncate(seq_id, min(self.cache.length(seq_id), keep))

    def release(self, seq_id) -> None:
        self.cache.free(seq_id)


class NoisyDraft(ModelDraft):
    """The noisy-copy drafter of BASELINE config 2's second variant (no counterpart in the
    reference): ModelDraft whose model is the target, with sigma * z added to each step's
    logits before probabilities(), z from oracle.noise at (seed, sequence id, position of the
    predicted token)."""

    def __init__(self, w: dict, prec: fw.Precision, num_blocks: int, block_size: int, sigma: float,
                 seed: int = 0) -> None:
        super().__init__(w, prec, num_blocks, block_size)
        self.sigma, self.seed = float(sigma), int(seed)

    def _logits(self, seq_ids, pending) -> np.ndarray:
        logits = super()._logits(seq_ids, pending)
        positions = [self.cache.length(s) for s in seq_ids]  # after the forward: past + n_new
        return noise.add_noise(logits, self.seed, self.sigma, seq_ids, positions)


def new_stats(k: int) -> dict:
    return dict(k=k, rounds=0, drafted=0, accepted=0, attempts=[0] * k, accepts=[0] * k, emitted_per_round=[],
                drafted_per_round=[])


def generate(w: dict, prec: fw.Precision, drafter, prompts: list[list[int]], max_new_tokens: int, k: int,
             temperature: float = 0.0, generator: torch.Generator | None = None, eos_id: int | None = None,
             num_blocks: int = 4096, block_size: int = 16, max_rounds: int | None = None):
    """spec/loop.py:38-104. Returns (outputs, stats dict). max_rounds bounds a CPU-baseline
    sample (None runs to completion)."""
    import time

    t_start = time.perf_counter()
    generator = generator or torch.Generator().manual_seed(0)
    cache = fw.Cache(w, num_blocks, block_size, prec)
    stats = new_stats(k)
    seq_ids = list(range(len(prompts)))
    for s in seq_ids:
        cache.add(s)
    first = sample(acc.probabilities(run(w, cache, seq_ids, prompts, prec).astype(np.float32), temperature),
                   generator).tolist()
    drafter.prefill(seq_ids, prompts)
    t_rounds = time.perf_counter()
    stats["seconds_prefill"] = t_rounds - t_start
    contexts = [p + [t] for p, t in zip(prompts, first)]
    outputs = [[t] for t in first]

    def finished(out):
        return len(out) >= max_new_tokens or (eos_id is not None and out[-1] == eos_id)

    def release(s):
        cache.free(s)
        drafter.release(s)

    active = [s for s in seq_ids if not finished(outputs[s])]
    for s in seq_ids:
        if s not in active:
            release(s)
    while active and (max_rounds is None or stats["rounds"] < max_rounds):
        ctx = [contexts[s] for s in active]
        draft, q = drafter.propose(active, ctx, k, temperature, generator)
        for s, c in zip(active, ctx):
            if cache.length(s) != len(c) - 1:
                raise RuntimeError(f"seq {s}: target cache holds {cache.length(s)}, expected {len(c) - 1}")
        ids = np.concatenate([np.array([[c[-1]] for c in ctx]), draft], axis=1)
        logits = fw.forward(w, cache, active, ids, [k + 1] * len(active), prec)
        p = acc.probabilities(logits.astype(np.float32), temperature)
        b = len(active)
        u_acc, u_res = _rand((b, k), generator), _rand((b,), generator)
        n_acc, nxt = acc.accept_reject(p, q, draft, u_acc, u_res)
        stats["rounds"] += 1
        still = []
        for row, s in enumerate(active):
            n = int(n_acc[row])
            stats["drafted"] += k
            stats["accepted"] += n
            for i in range(min(n + 1, k)):
                stats["attempts"][i] += 1
            for i in range(n):
                stats["accepts"][i] += 1
            new = [int(x) for x in draft[row, :n]] + [int(nxt[row])]
            new = new[: max_new_tokens - len(outputs[s])]
            if eos_id is not None and eos_id in new:
                new = new[: new.index(eos_id) + 1]
            stats["emitted_per_round"].append(len(new))
            stats["drafted_per_round"].append(min(n, len(new)))
            before = len(contexts[s])
            contexts[s] = contexts[s] + new
            outputs[s] = outputs[s] + new
            if finished(outputs[s]):
                release(s)
                continue
            cache.truncate(s, before + n)
            drafter.rollback(s, before + n)
            still.append(s)
        active = still
    stats["seconds_rounds"] = time.perf_counter() - t_rounds
    return outputs, stats


def generate_plain(w: dict, prec: fw.Precision, prompt: list[int], max_new_tokens: int, eos_id: int | None = None,
                   num_blocks: int = 4096, block_size: int = 16) -> list[int]:
    """baselines/cached_autoregressive.py:11-39 at temperature 0 (argmax, first maximum)."""
    cache = fw.Cache(w, num_blocks, block_size, prec)
    cache.add(0)
    logits = fw.forward(w, cache, [0], np.array([prompt]), [len(prompt)], prec, last_only=True)[0]
    out: list[int] = []
    for _ in range(max_new_tokens):
        tok = int(np.argmax(logits))
        out.append(tok)
        if tok == eos_id or len(out) == max_new_tokens:
            break
        logits = fw.forward(w, cache, [0], np.array([[tok]]), [1], prec)[0, 0]
    return out
