"""Oracle: probabilities + accept-reject + residual + inverse-CDF sampling, in numpy.

Restates lm/sampling.py:13-18 and spec/accept.py:18-79 of the reference. Computation is in
the input dtype (float32 unless the caller passes float64), with the reference's order of
operations: softmax as exp(z - max) * (1 / sum), acceptance as u * q_x < p_x, n as the
length of the leading run of acceptances, the bonus row as a rejection against a zero q row,
and sampling as the first index whose cumulative sum exceeds u * total (searchsorted with
right=True), clamped to V - 1. The cumulative sum accumulates in float64 and rounds each
prefix to the input dtype, as torch's CPU cumsum does for float32.
"""
from __future__ import annotations

import numpy as np


def probabilities(logits: np.ndarray, temperature: float) -> np.ndarray:
    """lm/sampling.py:13-18."""
    x = np.asarray(logits, dtype=np.float32)
    if temperature == 0.0:
        out = np.zeros_like(x)
        idx = np.argmax(x, axis=-1)
        np.put_along_axis(out, idx[..., None], 1.0, axis=-1)
        return out
    z = x / np.float32(temperature)
    e = np.exp(z - z.max(axis=-1, keepdims=True)).astype(np.float32)
    s = e.sum(axis=-1, keepdims=True, dtype=np.float32)
    return (e * (np.float32(1.0) / s)).astype(np.float32)


def residual_distribution(p: np.ndarray, q: np.ndarray) -> np.ndarray:
    """spec/accept.py:18-26: norm(max(0, p - q)), or p where that sums to 0."""
    r = np.maximum(p - q, 0.0).astype(p.dtype)
    total = r.sum(axis=-1, keepdims=True, dtype=p.dtype)
    tiny = np.finfo(p.dtype).tiny
    return np.where(total > 0, r / np.maximum(total, tiny), p).astype(p.dtype)


def sample_inverse_cdf(probs: np.ndarray, u: np.ndarray) -> np.ndarray:
    """spec/accept.py:29-35."""
    probs = np.asarray(probs)
    cdf = np.cumsum(probs.astype(np.float64), axis=-1).astype(probs.dtype)
    target = (np.asarray(u, dtype=probs.dtype) * cdf[:, -1])[:, None]
    idx = (cdf <= target).sum(axis=-1)  # searchsorted(right=True) on a non-decreasing cdf
    return np.minimum(idx, probs.shape[-1] - 1).astype(np.int64)


def accept_reject(p: np.ndarray, q: np.ndarray, draft: np.ndarray, u_accept: np.ndarray,
                  u_residual: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """spec/accept.py:44-79 with explicit uniforms. p [B,k+1,V], q [B,k,V], draft [B,k]."""
    b, k = draft.shape
    rows = np.arange(b)
    p_x = np.take_along_axis(p[:, :k], draft[..., None], axis=-1)[..., 0]
    q_x = np.take_along_axis(q, draft[..., None], axis=-1)[..., 0]
    if not np.all(q_x > 0):
        raise ValueError("a drafted token has zero draft probability; q is not what it was sampled from")
    accepted = np.asarray(u_accept, dtype=p.dtype) * q_x < p_x
    n = np.cumprod(accepted.astype(np.int64), axis=-1).sum(axis=-1)
    # the bonus row is a zero-q row (spec/accept.py pads with zeros shaped like one q row; the
    # explicit shape also covers k = 0, the plain sampler: the residual of p and 0 is p)
    q_padded = np.concatenate([q, np.zeros((b, 1, p.shape[-1]), dtype=q.dtype)], axis=1)
    r = residual_distribution(p[rows, n], q_padded[rows, n])
    return n.astype(np.int64), sample_inverse_cdf(r, u_residual)


def accept_reject_logits(p_logits: np.ndarray, q_logits: np.ndarray | None, draft: np.ndarray, u_accept: np.ndarray,
                         u_residual: np.ndarray, temperature: float) -> tuple[np.ndarray, np.ndarray]:
    """probabilities() of both sides, then accept_reject: the fused kernel's logit mode.
    q_logits None means q is the one-hot of the draft (NGramDraft, spec/ngram.py:22-23)."""
    p = probabilities(p_logits, temperature)
    if q_logits is None:
        q = np.zeros((draft.shape[0], draft.shape[1], p.shape[-1]), dtype=np.float32)
        np.put_along_axis(q, draft[..., None], 1.0, axis=-1)
    else:
        q = probabilities(q_logits, temperature)
    return accept_reject(p, q, draft, u_accept, u_residual)
