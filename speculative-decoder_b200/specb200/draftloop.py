"""The draft model's k proposal steps as one device-resident launch sequence.

Semantics of spec/draft.py:42-56 (ModelDraft.propose): step 0 feeds every token the draft
cache has not seen yet (one, or two after a round in which all k drafts were accepted), each
later step feeds the token the previous step sampled; each step's distribution is
probabilities(logits, T) of the last fed position and its token the inverse-CDF sample under
one caller-drawn uniform per row.

On the engine a step is three launches on the current stream and nothing returns to the host
in between: the draft forward (last-token logits), the fused sampler (the accept kernel with
k = 0 in logit mode: softmax at T, or argmax at T = 0, then the inverse CDF at u) and a scatter
that writes the sampled token into column j of the draft and into the next step's input. The
logits of every step stay on the device, step-major [k, B, V], for the accept kernel (which
reads them as q in logit mode) or for probabilities().

The host prepares, before the launches, what the steps read: the pending tokens of step 0,
each step's past length and new-token count per row, the draft cache's block tables and the
uniforms, all in device buffers that `DraftSteps` owns or that a caller (the fused round)
hands it.

With `noise = (sigma, seed)` each step adds seeded N(0, sigma^2) noise to its logits before
the sampler reads them (specb200_logit_noise: Philox4x32-10 at (seed, row id, position of the
predicted token)), which makes the noisy-copy drafter of BASELINE config 2's second variant;
the stored q logits then include the noise, as the accept step must see them.
"""
from __future__ import annotations

import torch

from specb200 import _ffi
from specb200._ffi import lib, ptr, raise_for
from specb200.engine import Engine


class DraftSteps:
    """Device buffers and launches of k draft steps for B rows of a draft model.

    Inputs (device, written by the caller before `launch`): ids0 [B, 2] int32 (the pending
    tokens of step 0, left-aligned), past [k, B] and n_new [k, B] int32 (0 new tokens leaves a
    row alone), table [B, W] int32, u [k, B] fp32. Outputs: draft [B, k] int64 and q_logits
    [k, B, V] fp32. `status` holds one int32 word per launch that reports errors (2 per step).
    """

    def __init__(self, eng: Engine, cache, B: int, k: int, cap: int, temperature: float,
                 ids0: torch.Tensor | None = None, past: torch.Tensor | None = None, n_new: torch.Tensor | None = None,
                 table: torch.Tensor | None = None, u: torch.Tensor | None = None,
                 fwd_ws: torch.Tensor | None = None, acc_ws: torch.Tensor | None = None,
                 noise: tuple[float, int] | None = None) -> None:
        self.eng, self.cache, self.B, self.k, self.cap, self.T = eng, cache, B, k, cap, float(temperature)
        self.noise = noise
        dev = eng.device
        i32, i64, f32 = torch.int32, torch.int64, torch.float32
        W = -(-cap // cache.block_size)
        self.ids0 = ids0 if ids0 is not None else torch.zeros(B, 2, dtype=i32, device=dev)
        self.past = past if past is not None else torch.zeros(k, B, dtype=i32, device=dev)
        self.n_new = n_new if n_new is not None else torch.zeros(k, B, dtype=i32, device=dev)
        self.table = table if table is not None else torch.zeros(B, W, dtype=i32, device=dev)
        self.u = u if u is not None else torch.zeros(k, B, dtype=f32, device=dev)
        self.q_logits = torch.empty(k, B, eng.vocab, dtype=f32, device=dev)
        self.draft = torch.zeros(B, k, dtype=i64, device=dev)
        self.ids = torch.zeros(B, 1, dtype=i32, device=dev)
        self.tok = torch.zeros(B, dtype=i64, device=dev)
        self.n_out = torch.zeros(B, dtype=i64, device=dev)  # the sampler's (unused) accepted counts
        self.status = torch.zeros(2 * k, dtype=i32, device=dev)
        self.row_ids = torch.arange(B, dtype=i32, device=dev)  # the noise stream of each row
        ws = max(eng.workspace_bytes(B, 2, cap), eng.workspace_bytes(B, 1, cap))
        self.fwd_ws = fwd_ws if fwd_ws is not None and fwd_ws.numel() >= ws else torch.zeros(ws, dtype=torch.uint8,
                                                                                          device=dev)
        aws = lib().specb200_accept_workspace_bytes(B, 0)
        self.acc_ws = acc_ws if acc_ws is not None and acc_ws.numel() >= aws else torch.zeros(aws, dtype=torch.uint8,
                                                                                          device=dev)

    def launch(self, status: torch.Tensor | None = None) -> None:
        """The k steps on the current stream (capturable in a CUDA graph). `status`, if given,
        replaces the object's own status words (2 k int32)."""
        L, B, k = lib(), self.B, self.k
        st = self.status if status is None else status
        s = torch.cuda.current_stream(self.eng.device).cuda_stream
        for j in range(k):
            ids = self.ids0 if j == 0 else self.ids
            self.eng.forward_device(self.cache, ids, self.n_new[j], self.past[j], self.table, self.cap, True,
                                    self.q_logits[j], st[2 * j:2 * j + 1], self.fwd_ws)
            if self.noise is not None:
                sigma, seed = self.noise
                V = self.eng.vocab
                raise_for(L.specb200_logit_noise(ptr(self.q_logits[j]), B, V, V, ptr(self.past[j]), ptr(self.n_new[j]),
                                                 ptr(self.row_ids), seed, sigma, s), "specb200_logit_noise")
            rc = L.specb200_accept(ptr(self.q_logits[j]), None, None, None, ptr(self.u[j]), B, 0, self.eng.vocab,
                                   _ffi.ACCEPT_LOGITS, self.T, ptr(self.n_out), ptr(self.tok),
                                   ptr(st[2 * j + 1:2 * j + 2]), ptr(self.acc_ws), self.acc_ws.numel(), s)
            raise_for(rc, "specb200_accept (draft sampler)")
            raise_for(L.specb200_scatter_tokens(ptr(self.tok), B, k, j, ptr(self.draft), ptr(self.ids), s),
                      "specb200_scatter_tokens")

    def plan(self, rows: list[int], contexts: list[list[int]]) -> tuple[list[list[int]], list[list[int]], list[list[int]]]:
        """Grow the draft cache for the k steps of the given rows (row index = sequence id in
        the cache) in the reference's order: step 0 the pending tokens, then one per step.
        Returns per step the rows' past lengths and new-token counts, and the pending tokens of
        step 0 per row."""
        pending = [contexts[i][self.cache.length(s):] for i, s in enumerate(rows)]
        if any(not 1 <= len(p) <= 2 for p in pending):
            raise RuntimeError("the draft cache must lag each context by one or two tokens")
        past, new = [], []
        for j in range(self.k):
            grow = [len(p) for p in pending] if j == 0 else [1] * len(rows)
            past.append(self.cache.reserve(rows, grow))
            new.append(grow)
        return past, new, pending
