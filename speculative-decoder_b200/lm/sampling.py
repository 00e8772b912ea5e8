"""Sampling helpers (lm/sampling.py of the reference) on the device."""
from __future__ import annotations

import torch

from specb200 import ops


def next_token(logits: torch.Tensor, temperature: float, generator: torch.Generator | None) -> int:
    """logits [V]. Temperature 0: argmax, ties to the lowest id (the fused kernel's greedy
    mode). Otherwise softmax(logits / T) on the device, then torch.multinomial on the host with
    the caller's generator, so the plain-decode baseline draws the reference's exact stream
    (lm/sampling.py:4-10). Only the plain-decode baseline uses this; the speculative round
    samples inside the fused accept kernel."""
    row = logits.reshape(1, 1, -1)
    if temperature == 0.0:
        u = torch.zeros(1, device=row.device)
        _, tok = ops.accept(row, None, None, None, u, logits=True, temperature=0.0)
        return int(tok.item())
    probs = ops.probabilities(row, temperature)[0, 0]
    return int(torch.multinomial(probs.cpu(), 1, generator=generator))


def probabilities(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    """[..., V] logits -> fp32 probabilities; temperature 0 gives the one-hot of the argmax."""
    return ops.probabilities(logits, temperature)
