"""Oracle: the cached Llama forward in numpy (test infrastructure only).

Restates lm/forward.py:21-68 (mask, embed, rotary, per-layer norm / q,k,v / RoPE / cache
write / gather / attention / o_proj + residual / MLP + residual, last-token select) and
lm/forward.py:71-84 (fp32-or-wider head) of the reference, with the Hugging Face Llama
pieces it calls: LlamaRMSNorm (transformers/models/llama/modeling_llama.py:62-67),
rotate_half / apply_rotary_pos_emb (modeling_llama.py:139-168), LlamaMLP (modeling_llama.py:
182-183) and the SDPA math with the reference's boolean mask.

Three precisions: "f64" and "f32" compute in that dtype; "bf16" keeps fp32 arrays and rounds
to bfloat16 (round to nearest even) after every op whose torch output is bf16, as the
reference's bf16 path does. Matmuls accumulate in the array dtype. Two small pieces use torch's
CPU kernels so that their fp32 rounding is exactly the reference's: the rotary cos/sin tables
and the RMSNorm mean of squares.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle.paged import Allocator, Table


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    bias = ((bits >> 16) & 1) + np.uint32(0x7FFF)
    out = ((bits + bias) & np.uint32(0xFFFF0000)).view(np.float32)
    return np.where(np.isnan(x), x, out)


class Precision:
    def __init__(self, mode: str) -> None:
        assert mode in ("f64", "f32", "bf16")
        self.mode = mode
        self.dtype = np.float64 if mode == "f64" else np.float32

    def r(self, x: np.ndarray) -> np.ndarray:
        x = np.asarray(x, dtype=self.dtype)
        return round_bf16(x) if self.mode == "bf16" else x


def weights_from_model(model) -> dict:
    """numpy copy of an HF Llama's weights (fp64 for an fp64 model, else fp32 holding the
    model's exact values) plus the shapes the forward needs."""
    cfg = model.config
    wide = torch.float64 if model.dtype == torch.float64 else torch.float32
    t = lambda p: p.detach().to("cpu", wide).numpy().copy()  # noqa: E731
    core = model.model
    layers = []
    for L in core.layers:
        a, m = L.self_attn, L.mlp
        layers.append(dict(ln1=t(L.input_layernorm.weight), q=t(a.q_proj.weight), k=t(a.k_proj.weight),
                           v=t(a.v_proj.weight), o=t(a.o_proj.weight), ln2=t(L.post_attention_layernorm.weight),
                           gate=t(m.gate_proj.weight), up=t(m.up_proj.weight), down=t(m.down_proj.weight)))
    head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    return dict(embed=t(core.embed_tokens.weight), norm=t(core.norm.weight), head=t(model.lm_head.weight),
                layers=layers, n_heads=cfg.num_attention_heads, n_kv_heads=cfg.num_key_value_heads,
                head_dim=head_dim, eps=float(cfg.rms_norm_eps),
                inv_freq=core.rotary_emb.inv_freq.detach().float().cpu().numpy().copy(),
                rope_scaling=float(getattr(core.rotary_emb, "attention_scaling", 1.0)))


def rope(w: dict, positions: np.ndarray, prec: Precision) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin [N, d] as LlamaRotaryEmbedding.forward computes them (fp32), cast to the
    activation precision (modeling_llama.py:124-135)."""
    inv = torch.from_numpy(w["inv_freq"]).float()
    pos = torch.from_numpy(np.asarray(positions, dtype=np.float32))
    freqs = (inv[:, None] @ pos[None, :]).t()
    emb = torch.cat([freqs, freqs], dim=-1)
    cos = (emb.cos() * w["rope_scaling"]).numpy()
    sin = (emb.sin() * w["rope_scaling"]).numpy()
    return prec.r(cos), prec.r(sin)


class Cache:
    """Paged K/V pool [n_layers, num_blocks * block_size, Hkv, d] + block tables."""

    def __init__(self, w: dict, num_blocks: int, block_size: int, prec: Precision) -> None:
        n_layers = len(w["layers"])
        self.bs = block_size
        self.k = np.zeros((n_layers, num_blocks * block_size, w["n_kv_heads"], w["head_dim"]), dtype=prec.dtype)
        self.v = np.zeros_like(self.k)
        self.alloc = Allocator(num_blocks)
        self.tables: dict[int, Table] = {}

    def add(self, s: int) -> None:
        if s in self.tables:
            raise ValueError(f"sequence {s} already present")
        self.tables[s] = Table()

    def free(self, s: int) -> None:
        self.tables[s].shrink_to(0, self.alloc, self.bs)
        del self.tables[s]

    def length(self, s: int) -> int:
        return self.tables[s].length

    def truncate(self, s: int, length: int) -> None:
        self.tables[s].shrink_to(length, self.alloc, self.bs)


def rmsnorm(x: np.ndarray, weight: np.ndarray, eps: float, prec: Precision) -> np.ndarray:
    """modeling_llama.py:62-67: the variance and the normalisation in fp32 whatever the
    activation dtype (the module casts to float32 first), cast back to the activation dtype,
    then weight * x_normed in that dtype. The fp32 mean of squares is reduced by torch's CPU
    kernel, so its rounding is the reference's own (a numpy pairwise sum differs in the last
    fp32 bit, which shows up at 1e-8 in fp64 logits)."""
    xt = torch.from_numpy(np.ascontiguousarray(x)).to(torch.float32)
    var = xt.pow(2).mean(-1, keepdim=True)
    normed = prec.r((xt * torch.rsqrt(var + eps)).numpy().astype(prec.dtype))
    return prec.r(weight.astype(prec.dtype) * normed)


def rotate_half(x: np.ndarray) -> np.ndarray:
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def forward(w: dict, cache: Cache, seq_ids: list[int], input_ids: np.ndarray, n_new: list[int], prec: Precision,
            last_only: bool = False) -> np.ndarray:
    """lm/forward.py:21-68 + logits(): returns [B, T, V] (or [B, V]) logits in fp32, or fp64
    in "f64" mode."""
    ids = np.asarray(input_ids, dtype=np.int64)
    b, t = ids.shape
    hq, hkv, d = w["n_heads"], w["n_kv_heads"], w["head_dim"]
    g = hq // hkv
    bs = cache.bs
    past = [cache.tables[s].length for s in seq_ids]
    for s, n in zip(seq_ids, n_new):
        tab = cache.tables[s]
        tab.grow_to(tab.length + n, cache.alloc, bs)
    total = [p + n for p, n in zip(past, n_new)]
    positions = np.array([[p + j for j in range(t)] for p in past])
    cos, sin = rope(w, positions.reshape(-1), prec)
    cos = cos.reshape(b, t, 1, d)
    sin = sin.reshape(b, t, 1, d)
    hidden = prec.r(w["embed"][ids])
    scale = d ** -0.5
    for li, L in enumerate(w["layers"]):
        x = rmsnorm(hidden, L["ln1"], w["eps"], prec)
        q = prec.r(x @ L["q"].T).reshape(b, t, hq, d)
        k = prec.r(x @ L["k"].T).reshape(b, t, hkv, d)
        v = prec.r(x @ L["v"].T).reshape(b, t, hkv, d)
        q = prec.r(prec.r(q * cos) + prec.r(rotate_half(q) * sin))
        k = prec.r(prec.r(k * cos) + prec.r(rotate_half(k) * sin))
        out = np.zeros((b, t, hq, d), dtype=prec.dtype)
        for bi, s in enumerate(seq_ids):
            tab = cache.tables[s]
            wslots = tab.slots(past[bi], total[bi], bs)
            cache.k[li][wslots] = k[bi, : n_new[bi]]
            cache.v[li][wslots] = v[bi, : n_new[bi]]
            rslots = tab.slots(0, total[bi], bs)
            acc = np.float64 if prec.mode == "f64" else np.float32
            kk = np.repeat(cache.k[li][rslots].astype(acc), g, axis=1)  # [S, Hq, d]: query head h reads kv head h // g
            vv = np.repeat(cache.v[li][rslots].astype(acc), g, axis=1)
            sc = np.einsum("thd,shd->hts", q[bi].astype(acc), kk) * acc(scale)
            allowed = np.arange(total[bi])[None, :] <= (past[bi] + np.arange(t))[:, None]  # key j <= query position
            sc = np.where(allowed[None], sc, -np.inf)
            e = np.exp(sc - sc.max(axis=-1, keepdims=True))
            pr = e / e.sum(axis=-1, keepdims=True)
            out[bi] = prec.r(np.einsum("hts,shd->thd", pr, vv))
        attn = out.reshape(b, t, hq * d)
        hidden = prec.r(hidden + prec.r(attn @ L["o"].T))
        x2 = rmsnorm(hidden, L["ln2"], w["eps"], prec)
        gate = prec.r(x2 @ L["gate"].T)
        up = prec.r(x2 @ L["up"].T)
        act = prec.r(prec.r(gate / (1 + np.exp(-gate))) * up)
        hidden = prec.r(hidden + prec.r(act @ L["down"].T))
    if last_only:
        hidden = hidden[np.arange(b), np.array(total) - np.array(past) - 1]
    hidden = rmsnorm(hidden, w["norm"], w["eps"], prec)
    wide = np.float64 if prec.mode == "f64" else np.float32
    return hidden.astype(wide) @ w["head"].astype(wide).T
