"""Prompt-lookup drafting (Saxena 2023) on the B200 (reference spec/ngram.py:4-45).

`lookup` and `NGramDraft.propose` run the warp-parallel n-gram kernel (specb200_ngram): for
n = min(max_n, len-1) down to 1, the most recent earlier occurrence of the last n tokens
wins, its continuation is copied forward (reading its own output once it runs past the end
of the context) and, with no match, the last token repeats. The result is bit-identical to
the reference's Python scan. The proposal is deterministic, so q is the one-hot of the
draft; the returned q carries a marker that lets accept_reject use the kernel's one-hot mode
instead of reading the V-wide rows.
"""
from __future__ import annotations

import torch

from specb200 import ops


def _device() -> torch.device:
    return torch.device("cuda", torch.cuda.current_device())


def contexts_tensor(contexts: list[list[int]], device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    width = max(1, max(len(c) for c in contexts))
    host = torch.zeros(len(contexts), width, dtype=torch.int32)
    for i, c in enumerate(contexts):
        if c:
            host[i, : len(c)] = torch.tensor(c, dtype=torch.int32)
    lens = torch.tensor([len(c) for c in contexts], dtype=torch.int32)
    return host.to(device), lens.to(device)


def onehot_q(draft: torch.Tensor, vocab_size: int) -> torch.Tensor:
    q = torch.zeros(*draft.shape, vocab_size, dtype=torch.float32, device=draft.device)
    q.scatter_(-1, draft.unsqueeze(-1), 1.0)
    q._specb200_onehot = True
    return q


class NGramDraft:
    def __init__(self, vocab_size: int, max_n: int = 3) -> None:
        self.vocab_size = vocab_size
        self.max_n = max_n

    def prefill(self, seq_ids: list[int], prompts: list[list[int]]) -> None:
        pass

    def propose(self, seq_ids: list[int], contexts: list[list[int]], k: int, temperature: float,
                generator: torch.Generator) -> tuple[torch.Tensor, torch.Tensor]:
        ctx, lens = contexts_tensor(contexts, _device())
        draft = ops.ngram(ctx, lens, k, self.max_n)
        return draft, onehot_q(draft, self.vocab_size)

    def rollback(self, seq_id: int, keep: int) -> None:
        pass

    def release(self, seq_id: int) -> None:
        pass


def lookup(context: list[int], k: int, max_n: int) -> list[int]:
    if not context:
        raise IndexError("lookup: empty context")
    ctx, lens = contexts_tensor([context], _device())
    return ops.ngram(ctx, lens, k, max_n)[0].tolist()
