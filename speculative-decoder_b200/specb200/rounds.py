"""Device-resident speculative rounds, replayed from one CUDA graph per generate() call.

spec.loop.generate takes this path for the engine's own drafters (NGramDraft, ModelDraft)
when `verify` and `accept_reject` are the engine's. The semantics are the reference's
(spec/loop.py:38-104; spec/draft.py:42-56; spec/ngram.py:19-23; spec/verify.py:9-30;
spec/accept.py:44-79); what changes is where the work runs:

  host, per round      grow the block tables (target: k+1 positions; draft: the lag
                       tokens, then one per step, in the reference's order), draw the round's
                       uniforms from the caller's generator in the reference's order, write
                       them and the tables into pinned buffers, replay the graph, wait, and
                       book the 3 small integers per row it returns (SpecStats, eos/budget
                       trimming, cache.truncate + drafter.rollback: spec/loop.py:79-100).
  device, one graph    H2D of the pinned inputs -> draft (n-gram kernel on the device-resident
                       contexts, or k draft-model forwards each followed by the fused sampler)
                       -> verify input ids, past lengths -> the (k+1)-token target forward ->
                       fused softmax + accept-reject + residual/bonus sample on the logits ->
                       context commit -> D2H of (n_accepted, next_token, draft, status).

Finished rows stay in the batch with n_new = 0 (no K/V writes, no attention, results
ignored), so the graph keeps one shape for the whole call. Every buffer the graph touches is
allocated before capture and lives as long as the round object.
"""
from __future__ import annotations

import torch

from specb200 import _ffi
from specb200._ffi import lib, ptr, raise_for
from specb200.draftloop import DraftSteps
from specb200.engine import Engine, engine_for


def fused_path_available(drafter, verify_fn, accept_fn) -> bool:
    from spec.accept import accept_reject
    from spec.draft import ModelDraft
    from spec.ngram import NGramDraft
    from spec.verify import verify

    if verify_fn is not verify or accept_fn is not accept_reject:
        return False
    if not torch.cuda.is_available():
        return False
    if type(drafter) is NGramDraft:
        return 1 <= drafter.max_n <= 8
    return type(drafter) is ModelDraft


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class FusedRound:
    """Buffers + captured graph for one (target, drafter, B, k, capacity)."""

    def __init__(self, target: Engine, cache, drafter, draft: Engine | None, B: int, k: int, cap: int,
                 temperature: float) -> None:
        self.t, self.cache, self.drafter, self.d = target, cache, drafter, draft
        self.B, self.k, self.cap, self.T = B, k, cap, float(temperature)
        self.V = target.vocab
        dev = target.device
        self.dev = dev
        i32, i64, f32 = torch.int32, torch.int64, torch.float32
        self.wt = -(-cap // cache.block_size)
        # ---- per-round host inputs, packed into one int32 and one float32 pinned buffer
        d_ints = 0
        if draft is not None:
            self.wd = -(-cap // drafter.cache.block_size)
            d_ints = B * 2 + 2 * k * B + B * self.wd
        n_ints = B + B * self.wt + d_ints
        n_flts = B * k + B + (k * B if draft is not None else 0)
        self.h_int = torch.zeros(n_ints, dtype=i32, pin_memory=True)
        self.h_flt = torch.zeros(n_flts, dtype=f32, pin_memory=True)
        self.g_int = torch.zeros(n_ints, dtype=i32, device=dev)
        self.g_flt = torch.zeros(n_flts, dtype=f32, device=dev)
        o = 0
        self.active_h, self.active = self.h_int[o:o + B], self.g_int[o:o + B]
        o += B
        self.table_h = self.h_int[o:o + B * self.wt].view(B, self.wt)
        self.table = self.g_int[o:o + B * self.wt].view(B, self.wt)
        o += B * self.wt
        if draft is not None:
            self.d_ids0_h = self.h_int[o:o + 2 * B].view(B, 2)
            self.d_ids0 = self.g_int[o:o + 2 * B].view(B, 2)
            o += 2 * B
            self.d_past_h = self.h_int[o:o + k * B].view(k, B)
            self.d_past = self.g_int[o:o + k * B].view(k, B)
            o += k * B
            self.d_n_h = self.h_int[o:o + k * B].view(k, B)
            self.d_n = self.g_int[o:o + k * B].view(k, B)
            o += k * B
            self.d_table_h = self.h_int[o:o + B * self.wd].view(B, self.wd)
            self.d_table = self.g_int[o:o + B * self.wd].view(B, self.wd)
        o = 0
        self.u_acc_h, self.u_acc = self.h_flt[o:o + B * k].view(B, k), self.g_flt[o:o + B * k].view(B, k)
        o += B * k
        self.u_res_h, self.u_res = self.h_flt[o:o + B], self.g_flt[o:o + B]
        o += B
        if draft is not None:
            self.d_u_h, self.d_u = self.h_flt[o:o + k * B].view(k, B), self.g_flt[o:o + k * B].view(k, B)
        # ---- device state
        self.ctx = torch.zeros(B, cap, dtype=i32, device=dev)
        self.ctx_len = torch.zeros(B, dtype=i32, device=dev)
        self.ids = torch.zeros(B, k + 1, dtype=i32, device=dev)
        self.past = torch.zeros(B, dtype=i32, device=dev)
        self.n_new = torch.zeros(B, dtype=i32, device=dev)
        self.p_logits = torch.empty(B, k + 1, self.V, dtype=f32, device=dev)
        self.n_acc = torch.zeros(B, dtype=i64, device=dev)
        self.nxt = torch.zeros(B, dtype=i64, device=dev)
        # one status word per launch that reports errors: draft forward + sampler per step,
        # n-gram, target forward, accept (a call clears its own word only)
        self.n_status = 2 * k + 3
        self.status = torch.zeros(self.n_status, dtype=i32, device=dev)
        # ---- outputs (pinned) and scratch
        self.out_h = torch.zeros(B * (2 + k), dtype=i64, pin_memory=True)
        self.status_h = torch.zeros(self.n_status, dtype=i32, pin_memory=True)
        self.out = torch.zeros(B * (2 + k), dtype=i64, device=dev)
        ws = target.workspace_bytes(B, k + 1, cap)
        if draft is not None:
            ws = max(ws, draft.workspace_bytes(B, 2, cap), draft.workspace_bytes(B, 1, cap))
        self.fwd_ws = torch.zeros(ws, dtype=torch.uint8, device=dev)
        acc_ws = max(lib().specb200_accept_workspace_bytes(B, k), lib().specb200_accept_workspace_bytes(B, 0))
        self.acc_ws = torch.zeros(acc_ws, dtype=torch.uint8, device=dev)
        # the draft model's k steps (the draft path), or the n-gram kernel's output buffer
        self.steps = None
        if draft is not None:
            self.steps = DraftSteps(draft, drafter.cache, B, k, cap, temperature, ids0=self.d_ids0, past=self.d_past,
                                    n_new=self.d_n, table=self.d_table, u=self.d_u, fwd_ws=self.fwd_ws,
                                    acc_ws=self.acc_ws, noise=drafter.noise())
            self.draft = self.steps.draft
        else:
            self.draft = torch.zeros(B, k, dtype=i64, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        # numpy views of the pinned inputs: the host fills them with plain array writes
        self.np_active = self.active_h.numpy()
        self.np_table = self.table_h.numpy()
        self.np_u_acc = self.u_acc_h.numpy()
        self.np_u_res = self.u_res_h.numpy()
        if draft is not None:
            self.np_d_ids0 = self.d_ids0_h.numpy()
            self.np_d_past = self.d_past_h.numpy()
            self.np_d_n = self.d_n_h.numpy()
            self.np_d_table = self.d_table_h.numpy()
            self.np_d_u = self.d_u_h.numpy()
        self.np_out = self.out_h.numpy()
        self.np_status = self.status_h.numpy()

    # ------------------------------------------------------------------ the round's launches
    def _launch(self) -> None:
        B, k, L = self.B, self.k, lib()
        s = _stream()
        self.g_int.copy_(self.h_int, non_blocking=True)
        self.g_flt.copy_(self.h_flt, non_blocking=True)
        st = self.status
        if self.steps is not None:
            self.steps.launch(st[0:2 * k])
        else:
            raise_for(L.specb200_ngram(ptr(self.ctx), self.cap, ptr(self.ctx_len), B, k, self.drafter.max_n,
                                       ptr(self.draft), ptr(st[0:1]), s), "specb200_ngram")
        raise_for(L.specb200_verify_ids(ptr(self.ctx), self.cap, ptr(self.ctx_len), ptr(self.draft), ptr(self.active), B,
                                        k, ptr(self.ids), ptr(self.past), ptr(self.n_new), s), "specb200_verify_ids")
        self.t.forward_device(self.cache, self.ids, self.n_new, self.past, self.table, self.cap, False, self.p_logits,
                              st[2 * k:2 * k + 1], self.fwd_ws)
        flags = _ffi.ACCEPT_LOGITS | (_ffi.ACCEPT_Q_STEP_MAJOR if self.d is not None else _ffi.ACCEPT_Q_ONEHOT)
        q = self.steps.q_logits if self.steps is not None else None
        rc = L.specb200_accept(ptr(self.p_logits), ptr(q), ptr(self.draft), ptr(self.u_acc), ptr(self.u_res), B, k,
                               self.V, flags, self.T, ptr(self.n_acc), ptr(self.nxt), ptr(st[2 * k + 1:2 * k + 2]),
                               ptr(self.acc_ws),
                               self.acc_ws.numel(), s)
        raise_for(rc, "specb200_accept")
        raise_for(L.specb200_commit_tokens(ptr(self.ctx), self.cap, ptr(self.ctx_len), ptr(self.draft), ptr(self.n_acc),
                                           ptr(self.nxt), ptr(self.active), B, k, s), "specb200_commit_tokens")
        self.out[0:B].copy_(self.n_acc)
        self.out[B:2 * B].copy_(self.nxt)
        self.out[2 * B:].copy_(self.draft.reshape(-1))
        self.out_h.copy_(self.out, non_blocking=True)
        self.status_h.copy_(st, non_blocking=True)

    def run(self) -> tuple[list[int], list[int], list[list[int]]]:
        if self.graph is None:
            main = torch.cuda.current_stream(self.dev)
            side = torch.cuda.Stream(self.dev)
            side.wait_stream(main)
            g = torch.cuda.CUDAGraph()
            # Captured with capture_begin/capture_end rather than the torch.cuda.graph() context:
            # that context first returns every cached device block and every cached pinned host
            # block to the driver, so each generate() call would re-allocate its KV pools and
            # pinned round buffers through cudaMalloc / cudaHostAlloc, which on B200 hosts
            # sporadically stalls a request for 60-570 ms.
            with torch.cuda.stream(side):
                g.capture_begin()
                try:
                    self._launch()
                finally:
                    g.capture_end()
            main.wait_stream(side)
            self.graph = g
        self.graph.replay()
        torch.cuda.current_stream(self.dev).synchronize()
        if self.np_status.any():
            code = int(self.np_status[self.np_status != 0][0])
            self.status.zero_()
            _ffi.check_status(torch.tensor([code]), "fused round")
        B, k = self.B, self.k
        vals = self.np_out.tolist()
        return vals[0:B], vals[B:2 * B], [vals[2 * B + b * k: 2 * B + (b + 1) * k] for b in range(B)]


def generate_fused(target, cache, drafter, prompts, max_new_tokens, k, temperature, generator, eos_id, on_event):
    from spec.draft import ModelDraft
    from spec.loop import SpecStats, finished, release, settle_row

    eng = engine_for(target)
    dev = eng.device
    B = len(prompts)
    stats = SpecStats(k)
    seq_ids = list(range(B))
    for s in seq_ids:
        cache.add(s)
    # Target prefill and the first token (spec/loop.py:61): the fused sampler on last-token logits.
    width = max(len(p) for p in prompts)
    ids = torch.tensor([p + [0] * (width - len(p)) for p in prompts], dtype=torch.int64)
    logits0 = eng.forward(cache, seq_ids, ids, [len(p) for p in prompts], last_only=True)
    u0 = torch.rand(B, generator=generator, dtype=torch.float32)
    from specb200 import ops

    _, first_t = ops.accept(logits0.view(B, 1, eng.vocab), None, None, None, u0.to(dev), logits=True,
                            temperature=temperature)
    first = first_t.tolist()
    on_event("first_token")
    drafter.prefill(seq_ids, prompts)
    on_event("draft_prefilled")
    contexts = [p + [t] for p, t in zip(prompts, first)]
    outputs = [[t] for t in first]
    active = [s for s in seq_ids if not finished(outputs[s], max_new_tokens, eos_id)]
    for s in seq_ids:
        if s not in active:
            release(cache, drafter, s)
    if not active:
        return outputs, stats

    draft_eng = engine_for(drafter.model) if isinstance(drafter, ModelDraft) else None
    if draft_eng is not None and draft_eng.vocab != eng.vocab:
        raise ValueError(f"draft vocab {draft_eng.vocab} != target vocab {eng.vocab}")
    cap = width + max_new_tokens + k + 2
    rnd = FusedRound(eng, cache, drafter, draft_eng, B, k, cap, temperature)
    for b, c in enumerate(contexts):
        rnd.ctx[b, : len(c)] = torch.tensor(c, dtype=torch.int32)
    rnd.ctx_len.copy_(torch.tensor([len(c) for c in contexts], dtype=torch.int32))

    while active:
        n_act = len(active)
        rnd.np_active[:] = 0
        rnd.np_active[active] = 1
        # uniforms in the reference's order: draft steps (ModelDraft.propose), then accept_reject
        if draft_eng is not None:
            d_u = [torch.rand(n_act, generator=generator, dtype=torch.float32).numpy() for _ in range(k)]
        rnd.np_u_acc[active] = torch.rand(n_act, k, generator=generator, dtype=torch.float32).numpy()
        rnd.np_u_res[active] = torch.rand(n_act, generator=generator, dtype=torch.float32).numpy()
        # draft cache: the lag tokens, then one per step, grown row by row as the reference does
        if draft_eng is not None:
            dc = drafter.cache
            rnd.np_d_n[:] = 0
            past, grow, pending = rnd.steps.plan(active, [contexts[s] for s in active])
            for j in range(k):
                rnd.np_d_u[j, active] = d_u[j]
                rnd.np_d_past[j, active] = past[j]
                rnd.np_d_n[j, active] = grow[j]
            for s, pend in zip(active, pending):
                rnd.np_d_ids0[s, : len(pend)] = pend
            for s in active:
                blocks = dc.tables[s].blocks
                rnd.np_d_table[s, : len(blocks)] = blocks
        # target cache: k + 1 positions past len(context) - 1 (the verify forward's append)
        for s in active:
            if cache.length(s) != len(contexts[s]) - 1:
                raise RuntimeError(f"seq {s}: target cache holds {cache.length(s)}, expected {len(contexts[s]) - 1}")
        cache.reserve(active, [k + 1] * n_act)
        for s in active:
            blocks = cache.tables[s].blocks
            rnd.np_table[s, : len(blocks)] = blocks

        n_acc, nxt, drafts = rnd.run()
        stats.rounds += 1
        active = [s for s in active
                  if settle_row(stats, cache, drafter, s, int(n_acc[s]), drafts[s], int(nxt[s]), contexts, outputs,
                                max_new_tokens, eos_id)]
        if stats.rounds == 1:
            on_event("first_round")
    return outputs, stats
