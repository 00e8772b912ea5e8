"""Speculative-sampling acceptance (Leviathan et al. 2023; Chen et al. 2023) on the B200.

Same interface and meaning as the reference's spec/accept.py:18-79. Draft token x_i ~ q_i is
accepted iff u_i * q_i(x_i) < p_i(x_i); n = the number of leading acceptances; the token
after them is one inverse-CDF sample from norm(max(0, p_n - q_n)), where the bonus row n = k
uses q = 0, and an all-zero residual falls back to p_n. All of it runs in one kernel
(specb200_accept); uniforms that are not given are drawn from the caller's generator in the
reference's order and dtype, so a seeded run consumes the generator exactly as the reference
does. Results come back on the device the inputs came from.

The kernel computes in fp32. fp64 inputs (as in the reference's fraction tests) are rounded
to fp32 first; the decision u*q < p can then only differ where the two sides are within fp32
rounding of each other.
"""
from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch

from specb200 import ops

Residual = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


def residual_distribution(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """norm(max(0, p - q)) over the last dim, or p where that has no mass. The fused kernel
    computes this itself; the function is the reference's residual hook (spec/accept.py:18-26)
    for callers that pass a `residual` of their own."""
    r = torch.clamp(p - q, min=0.0)
    total = r.sum(dim=-1, keepdim=True)
    return torch.where(total > 0, r / total.clamp(min=torch.finfo(r.dtype).tiny), p)


def _cuda_device(t: torch.Tensor) -> torch.device:
    return t.device if t.device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())


def sample_inverse_cdf(probs: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """probs [B, V] (need not sum to 1), u [B] in [0, 1): token i is chosen iff u * total lies
    in [cdf[i-1], cdf[i]), so zero-probability tokens are never chosen (spec/accept.py:29-35)."""
    dev = _cuda_device(probs)
    p = probs.to(dev).float().unsqueeze(1)
    _, tok = ops.accept(p, None, None, None, u.to(dev), logits=False)
    return tok.to(probs.device)


@dataclass(frozen=True)
class Verdict:
    n_accepted: torch.Tensor  # [B] leading draft tokens kept, 0..k
    next_token: torch.Tensor  # [B] residual sample at the first rejection, or the bonus token


def draw_uniforms(b: int, k: int, generator: torch.Generator | None, dtype: torch.dtype,
                  device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """u_accept [b, k] then u_residual [b], in the reference's order (spec/accept.py:60-63),
    drawn where the generator lives."""
    where = generator.device if generator is not None else device
    u_accept = torch.rand(b, k, generator=generator, dtype=dtype, device=where)
    u_residual = torch.rand(b, generator=generator, dtype=dtype, device=where)
    return u_accept, u_residual


def accept_reject(
    p: torch.Tensor,
    q: torch.Tensor,
    draft: torch.Tensor,
    generator: torch.Generator | None = None,
    u_accept: torch.Tensor | None = None,
    u_residual: torch.Tensor | None = None,
    residual: Residual = residual_distribution,
) -> Verdict:
    """p [B, k+1, V] target probabilities, q [B, k, V] the draft distributions the draft
    tokens were sampled from, draft [B, k]. At temperature 0 both are one-hot and this is
    exact greedy verification."""
    b, k = draft.shape
    if u_accept is None or u_residual is None:
        ua, ur = draw_uniforms(b, k, generator, p.dtype, p.device)
        u_accept = ua if u_accept is None else u_accept
        u_residual = ur if u_residual is None else u_residual
    home = p.device
    dev = _cuda_device(p)
    onehot = bool(getattr(q, "_specb200_onehot", False))
    pd = p.to(dev)
    qd = None if onehot else q.to(dev)
    dd = draft.to(dev)
    if residual is residual_distribution:
        n, nxt = ops.accept(pd, qd, dd, u_accept.to(dev), u_residual.to(dev), logits=False, q_onehot=onehot)
        return Verdict(n.to(home), nxt.to(home))
    # A caller-supplied residual: the kernel decides n, the hook builds the distribution at
    # row n, and the kernel's sampler draws from it.
    n, _ = ops.accept(pd, qd, dd, u_accept.to(dev), u_residual.to(dev), logits=False, q_onehot=onehot,
                      decide_only=True)
    qfull = torch.nn.functional.one_hot(dd, pd.shape[-1]).to(pd.dtype) if onehot else qd.to(pd.dtype)
    q_padded = torch.cat([qfull, torch.zeros_like(pd[:, :1])], dim=1)
    rows = torch.arange(b, device=dev)
    r = residual(pd[rows, n], q_padded[rows, n])
    nxt = sample_inverse_cdf(r, u_residual.to(dev))
    return Verdict(n.to(home), nxt.to(home))
