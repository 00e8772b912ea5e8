"""Plain (non-speculative) greedy decoding on the engine: one CUDA-graph replay per token.

The semantics are those of the reference's cached decoding loop
(baselines/cached_autoregressive.py:11-90 with lm/sampling.py:4-10 at temperature 0): each
step feeds every running row's last token, appends one position to its cache, and takes the
first maximum of the last-token logits. What runs per token is one graph: the H2D copy of the
rows' past lengths, new-token counts and block tables from pinned memory, the engine forward
(T = 1, last-token logits), the fused sampler in greedy mode (the accept kernel with k = 0 at
temperature 0: the first argmax, as torch.argmax picks it), a scatter of the tokens into the
next step's input, and a D2H copy of the tokens into pinned memory. The host reads the tokens
after each replay (for eos and the output lists) and grows the block tables in the
reference's order; finished rows stay in the graph with no new tokens (no K/V writes, no
attention) so its shape never changes.
"""
from __future__ import annotations

import torch

from specb200 import _ffi
from specb200._ffi import lib, ptr, raise_for
from specb200.engine import Engine


class PlainDecoder:
    """Graph and buffers of greedy T = 1 steps for B rows (row b = cache sequence rows[b])."""

    def __init__(self, eng: Engine, cache, rows: list[int], cap: int) -> None:
        self.eng, self.cache, self.rows, self.cap = eng, cache, list(rows), cap
        B = len(rows)
        self.B = B
        dev = eng.device
        i32, i64, f32 = torch.int32, torch.int64, torch.float32
        W = -(-cap // cache.block_size)
        # pinned per-step inputs: past [B], n_new [B], table [B, W] in one buffer
        self.h_in = torch.zeros(2 * B + B * W, dtype=i32, pin_memory=True)
        self.g_in = torch.zeros_like(self.h_in, device=dev)
        self.np_past = self.h_in[:B].numpy()
        self.np_new = self.h_in[B:2 * B].numpy()
        self.np_table = self.h_in[2 * B:].view(B, W).numpy()
        self.past = self.g_in[:B]
        self.n_new = self.g_in[B:2 * B]
        self.table = self.g_in[2 * B:].view(B, W)
        self.ids = torch.zeros(B, 1, dtype=i32, device=dev)
        self.logits = torch.empty(B, eng.vocab, dtype=f32, device=dev)
        self.tok = torch.zeros(B, dtype=i64, device=dev)
        self.n_out = torch.zeros(B, dtype=i64, device=dev)
        self.u = torch.zeros(B, dtype=f32, device=dev)  # greedy: the sampler ignores it
        self.status = torch.zeros(2, dtype=i32, device=dev)
        self.tok_h = torch.zeros(B, dtype=i64, pin_memory=True)
        self.status_h = torch.zeros(2, dtype=i32, pin_memory=True)
        self.fwd_ws = torch.zeros(eng.workspace_bytes(B, 1, cap), dtype=torch.uint8, device=dev)
        self.acc_ws = torch.zeros(lib().specb200_accept_workspace_bytes(B, 0), dtype=torch.uint8, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None

    def _launch(self) -> None:
        s = torch.cuda.current_stream(self.eng.device).cuda_stream
        self.g_in.copy_(self.h_in, non_blocking=True)
        self.eng.forward_device(self.cache, self.ids, self.n_new, self.past, self.table, self.cap, True, self.logits,
                                self.status[0:1], self.fwd_ws)
        rc = lib().specb200_accept(ptr(self.logits), None, None, None, ptr(self.u), self.B, 0, self.eng.vocab,
                                   _ffi.ACCEPT_LOGITS, 0.0, ptr(self.n_out), ptr(self.tok), ptr(self.status[1:2]),
                                   ptr(self.acc_ws), self.acc_ws.numel(), s)
        raise_for(rc, "specb200_accept (greedy sampler)")
        raise_for(lib().specb200_scatter_tokens(ptr(self.tok), self.B, 1, 0, None, ptr(self.ids), s),
                  "specb200_scatter_tokens")
        self.tok_h.copy_(self.tok, non_blocking=True)
        self.status_h.copy_(self.status, non_blocking=True)

    def start(self, first: torch.Tensor) -> None:
        """The tokens the prefill produced, [B] on the device, become the first step's input."""
        self.ids.copy_(first.view(self.B, 1).to(torch.int32))

    def step(self, active: list[int]) -> list[int]:
        """One greedy token for each row index in `active` (the others are left alone)."""
        new = self.cache.reserve([self.rows[i] for i in active], [1] * len(active))
        self.np_new[:] = 0
        for i, p in zip(active, new):
            self.np_past[i] = p
            self.np_new[i] = 1
            blocks = self.cache.tables[self.rows[i]].blocks
            self.np_table[i, : len(blocks)] = blocks
        if self.graph is None:
            main = torch.cuda.current_stream(self.eng.device)
            side = torch.cuda.Stream(self.eng.device)
            side.wait_stream(main)
            g = torch.cuda.CUDAGraph()
            # capture_begin/capture_end keep torch's cached device and pinned blocks (the
            # torch.cuda.graph() context would first return them all to the driver)
            with torch.cuda.stream(side):
                g.capture_begin()
                try:
                    self._launch()
                finally:
                    g.capture_end()
            main.wait_stream(side)
            self.graph = g
        self.graph.replay()
        torch.cuda.current_stream(self.eng.device).synchronize()
        if self.status_h.any():
            code = int(self.status_h[self.status_h != 0][0])
            self.status.zero_()
            _ffi.check_status(torch.tensor([code]), "plain decode step")
        return self.tok_h.tolist()
