"""Torch-tensor wrappers of the C ABI: each takes CUDA tensors, checks shapes, launches on
the current stream and returns CUDA tensors. Used by the drop-in modules (spec/, lm/) and
by the layer-level parity tests."""
from __future__ import annotations

import torch

from specb200 import _ffi
from specb200._ffi import Workspace, lib, ptr, raise_for, stream_ptr


def _status(device: torch.device) -> torch.Tensor:
    return Workspace.get("status", 4, device)[:4].view(torch.int32)


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return _ffi.F32
    if dtype == torch.bfloat16:
        return _ffi.BF16
    raise NotImplementedError(f"the B200 engine runs float32 and bfloat16, not {dtype}")


def accept(p: torch.Tensor, q: torch.Tensor | None, draft: torch.Tensor, u_accept: torch.Tensor,
           u_residual: torch.Tensor, *, logits: bool, temperature: float = 1.0, q_onehot: bool = False,
           decide_only: bool = False, check: bool = True,
           out: tuple[torch.Tensor, torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused accept-reject (spec/accept.py:44-79, lm/sampling.py:13-18) on fp32 rows.
    p [B, k+1, V], q [B, k, V] or None (q_onehot, or k == 0), draft [B, k] int64."""
    _ffi.require_cuda(p, "accept")
    b, k1, v = p.shape
    k = k1 - 1
    dev = p.device
    p = p.contiguous().float()
    if q is not None and not q_onehot:
        q = q.to(dev).contiguous().float()
        if q.shape != (b, k, v):
            raise ValueError(f"accept: q has shape {tuple(q.shape)}, expected {(b, k, v)}")
    else:
        q = None
    draft = draft.to(dev, torch.int64).contiguous() if k > 0 else torch.zeros(b, 1, dtype=torch.int64, device=dev)
    u_accept = u_accept.to(dev, torch.float32).contiguous() if k > 0 else torch.zeros(b, 1, device=dev)
    u_residual = u_residual.to(dev, torch.float32).contiguous()
    if out is None:
        n_acc = torch.empty(b, dtype=torch.int64, device=dev)
        nxt = torch.empty(b, dtype=torch.int64, device=dev)
    else:
        n_acc, nxt = out
    flags = (_ffi.ACCEPT_LOGITS if logits else 0) | (_ffi.ACCEPT_Q_ONEHOT if q_onehot else 0) | \
            (_ffi.ACCEPT_DECIDE_ONLY if decide_only else 0)
    nbytes = lib().specb200_accept_workspace_bytes(b, k)
    ws = Workspace.get("accept", nbytes, dev)
    status = _status(dev)
    rc = lib().specb200_accept(ptr(p), ptr(q), ptr(draft), ptr(u_accept), ptr(u_residual), b, k, v, flags,
                               float(temperature), ptr(n_acc), ptr(nxt), ptr(status), ptr(ws), ws.numel(),
                               stream_ptr(dev))
    raise_for(rc, "specb200_accept")
    if check:
        _ffi.check_status(status, "accept")
    return n_acc, nxt


def probabilities(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    """lm/sampling.py:13-18 on the device: [..., V] logits -> fp32 probabilities."""
    _ffi.require_cuda(logits, "probabilities")
    x = logits.contiguous().float()
    v = x.shape[-1]
    rows = x.numel() // v
    out = torch.empty_like(x)
    rc = lib().specb200_probabilities(ptr(x), rows, v, float(temperature), ptr(out), stream_ptr(x.device))
    raise_for(rc, "specb200_probabilities")
    return out


def ngram(ctx: torch.Tensor, ctx_len: torch.Tensor, k: int, max_n: int, check: bool = True,
          out: torch.Tensor | None = None) -> torch.Tensor:
    """spec/ngram.py:32-45 for B contexts at once. ctx [B, stride] int32, ctx_len [B] int32."""
    _ffi.require_cuda(ctx, "ngram")
    b, stride = ctx.shape
    draft = out if out is not None else torch.empty(b, k, dtype=torch.int64, device=ctx.device)
    status = _status(ctx.device)
    rc = lib().specb200_ngram(ptr(ctx), stride, ptr(ctx_len), b, k, max_n, ptr(draft), ptr(status),
                              stream_ptr(ctx.device))
    raise_for(rc, "specb200_ngram")
    if check:
        _ffi.check_status(status, "ngram")
    return draft


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    _ffi.require_cuda(x, "rmsnorm")
    x = x.contiguous()
    h = x.shape[-1]
    y = torch.empty_like(x)
    rc = lib().specb200_rmsnorm(_dtype_code(x.dtype), ptr(x), ptr(weight.contiguous()), x.numel() // h, h, eps, ptr(y),
                                stream_ptr(x.device))
    raise_for(rc, "specb200_rmsnorm")
    return y


def linear(x: torch.Tensor, w: torch.Tensor, out_f32: bool = False) -> torch.Tensor:
    """x [M, K] @ w[N, K]^T; bf16 on tcgen05, fp32 on FFMA."""
    _ffi.require_cuda(x, "linear")
    x = x.contiguous()
    w = w.contiguous()
    m, kdim = x.shape
    n = w.shape[0]
    y = torch.empty(m, n, dtype=torch.float32 if out_f32 else x.dtype, device=x.device)
    nbytes = lib().specb200_linear_workspace_bytes(m, n, kdim)
    ws = Workspace.get("linear", nbytes, x.device)
    status = _status(x.device)
    rc = lib().specb200_linear(_dtype_code(x.dtype), ptr(w), ptr(x), m, n, kdim, int(out_f32), ptr(y), ptr(ws),
                               ws.numel(), ptr(status), stream_ptr(x.device))
    raise_for(rc, "specb200_linear")
    _ffi.check_status(status, "linear")
    return y


def attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, block_table: torch.Tensor,
              block_size: int, past_len: torch.Tensor, n_new: torch.Tensor, scale: float,
              max_kv_len: int) -> torch.Tensor:
    """q [B, T, Hq, d]; pools [num_slots, Hkv, d]; block_table [B, W] int32."""
    _ffi.require_cuda(q, "attention")
    b, t, hq, d = q.shape
    hkv = k_pool.shape[1]
    out = torch.empty_like(q)
    nbytes = lib().specb200_attention_workspace_bytes(b, t, hq, hkv, d, max_kv_len)
    ws = Workspace.get("attention", nbytes, q.device)
    status = _status(q.device)
    rc = lib().specb200_attention(_dtype_code(q.dtype), ptr(q.contiguous()), ptr(k_pool), ptr(v_pool),
                                  ptr(block_table), block_table.shape[1], block_size, ptr(past_len), ptr(n_new), b, t,
                                  hq, hkv, d, max_kv_len, scale, ptr(out), ptr(ws), ws.numel(), ptr(status),
                                  stream_ptr(q.device))
    raise_for(rc, "specb200_attention")
    _ffi.check_status(status, "attention")
    return out


def commit_tokens(ctx: torch.Tensor, ctx_len: torch.Tensor, draft: torch.Tensor, n_accepted: torch.Tensor,
                  next_token: torch.Tensor, active: torch.Tensor | None = None) -> None:
    b, stride = ctx.shape
    k = draft.shape[1]
    rc = lib().specb200_commit_tokens(ptr(ctx), stride, ptr(ctx_len), ptr(draft), ptr(n_accepted), ptr(next_token),
                                      ptr(active), b, k, stream_ptr(ctx.device))
    raise_for(rc, "specb200_commit_tokens")


def verify_ids(ctx: torch.Tensor, ctx_len: torch.Tensor, draft: torch.Tensor, out: torch.Tensor,
               active: torch.Tensor | None = None, past: torch.Tensor | None = None,
               n_new: torch.Tensor | None = None) -> torch.Tensor:
    b, stride = ctx.shape
    k = draft.shape[1]
    rc = lib().specb200_verify_ids(ptr(ctx), stride, ptr(ctx_len), ptr(draft), ptr(active), b, k, ptr(out), ptr(past),
                                   ptr(n_new), stream_ptr(ctx.device))
    raise_for(rc, "specb200_verify_ids")
    return out
