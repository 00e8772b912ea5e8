"""Oracle: the seeded logit noise of the noisy-copy drafter (test infrastructure only).

BASELINE config 2's second variant drafts with the target itself plus N(0, sigma^2) noise on
its final logits; the reference has no such drafter, so both sides restate one definition.
The noise of a row at a position is a pure function of (seed, row id, position, vocabulary
index):

    (r0, r1, r2, r3) = Philox4x32-10(counter = (v, position, row_id, 0), key = (seed lo, seed hi))
    u1 = ((r0 >> 8) + 0.5) * 2^-24,  u2 = (r1 >> 8) * 2^-24
    z  = sqrt(-2 ln u1) * cos(2 pi u2)                (Box-Muller, computed in float32)

Philox4x32-10 is the counter-based generator of Salmon, Moraes, Dror and Shaw, "Parallel
random numbers: as easy as 1, 2, 3" (SC 2011), restated here in numpy with uint64 products.
Its known-answer vectors (from that paper's Random123 distribution) pin this restatement.
"""
from __future__ import annotations

import numpy as np

M0, M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
W0, W1 = 0x9E3779B9, 0xBB67AE85
MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0: int, k1: int) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Vectorised over the counter words (broadcastable uint32 arrays); returns four uint32 arrays."""
    c = [np.asarray(x, dtype=np.uint64) & MASK for x in np.broadcast_arrays(c0, c1, c2, c3)]
    k0, k1 = k0 & 0xFFFFFFFF, k1 & 0xFFFFFFFF
    for r in range(10):
        if r > 0:
            k0 = (k0 + W0) & 0xFFFFFFFF
            k1 = (k1 + W1) & 0xFFFFFFFF
        p0 = M0 * c[0]
        p1 = M1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK
        c = [hi1 ^ c[1] ^ np.uint64(k0), lo1, hi0 ^ c[3] ^ np.uint64(k1), lo0]
    return tuple(x.astype(np.uint32) for x in c)


def normals(seed: int, row_id: int, position: int, vocab: int) -> np.ndarray:
    """z [vocab] float32 for one row at one position."""
    v = np.arange(vocab, dtype=np.uint64)
    r0, r1, _, _ = philox4x32_10(v, position, row_id, 0, seed & 0xFFFFFFFF, seed >> 32)
    u1 = ((r0 >> np.uint32(8)).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -24)
    u2 = (r1 >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)
    return (np.sqrt(np.float32(-2.0) * np.log(u1)) * np.cos(np.float32(2.0 * np.pi) * u2)).astype(np.float32)


def add_noise(logits: np.ndarray, seed: int, sigma: float, row_ids, positions) -> np.ndarray:
    """logits [B, V] fp32 + sigma * z per row (row_ids[b], positions[b])."""
    out = np.array(logits, dtype=np.float32, copy=True)
    for b, (rid, pos) in enumerate(zip(row_ids, positions)):
        out[b] = (out[b] + np.float32(sigma) * normals(seed, int(rid), int(pos), out.shape[1])).astype(np.float32)
    return out
