"""The engine's view of a Hugging Face Llama/Qwen2 model: packed weights + the C model handle.

Packing (done once per model and cached, as the reference caches its fp32 head at
lm/forward.py:80-83):
  w_qkv      = cat(q_proj, k_proj, v_proj)                     [(Hq + 2 Hkv) d, H]
  w_gate_up  = 64-row groups, gate rows 64g..64g+63 then up rows [2 I, H]
               (a 128-row GEMM tile then holds the gate and up rows of the same 64 features,
               so SiLU(gate) * up is computed in that tile's epilogue)
  rope_cos/sin[pos, i] = cos/sin(pos * inv_freq[i]) * attention_scaling in fp32, computed on
               the host with torch exactly as LlamaRotaryEmbedding.forward does
               (transformers/models/llama/modeling_llama.py:124-135), for every position.
The K/V pool is the KVCache's own tensors; the forward writes new entries into their slots.
"""
from __future__ import annotations

import ctypes
import weakref

import torch

from specb200 import _ffi
from specb200._ffi import Workspace, lib, ptr, raise_for, stream_ptr

MIN_POSITIONS = 16384


def _packed_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    inter, hidden = gate.shape
    g = gate.reshape(inter // 64, 64, hidden)
    u = up.reshape(inter // 64, 64, hidden)
    return torch.stack([g, u], dim=1).reshape(2 * inter, hidden).contiguous()


class Engine:
    """Packed weights of one model on one CUDA device."""

    def __init__(self, model: torch.nn.Module) -> None:
        from lm.forward import check_supported

        check_supported(model)
        cfg = model.config
        core = model.model
        dtype = core.embed_tokens.weight.dtype
        if dtype not in (torch.float32, torch.bfloat16):
            raise NotImplementedError(f"the B200 engine runs float32 and bfloat16 models, not {dtype}")
        device = core.embed_tokens.weight.device
        if device.type != "cuda":
            raise RuntimeError(f"the B200 engine needs the model on a CUDA device (got {device}); there is no CPU path")
        self.device = device
        self.dtype = dtype
        self.n_layers = cfg.num_hidden_layers
        self.hidden = cfg.hidden_size
        self.n_heads = cfg.num_attention_heads
        self.n_kv_heads = cfg.num_key_value_heads
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.intermediate = cfg.intermediate_size
        self.vocab = cfg.vocab_size
        self.eps = float(cfg.rms_norm_eps)
        for layer in core.layers:
            a = layer.self_attn
            if a.o_proj.bias is not None or any(p.bias is not None for p in (a.q_proj, a.k_proj, a.v_proj)):
                raise NotImplementedError("attention projections with bias are not supported by the B200 engine")
            m = layer.mlp
            if any(p.bias is not None for p in (m.gate_proj, m.up_proj, m.down_proj)):
                raise NotImplementedError("MLP bias is not supported by the B200 engine")
        if self.intermediate % 64:
            raise NotImplementedError("intermediate_size must be a multiple of 64")
        if self.head_dim not in (16, 32, 64):
            raise NotImplementedError(f"head_dim {self.head_dim} is not supported (16, 32 or 64)")

        with torch.no_grad():
            self.layers = []
            for layer in core.layers:
                a, m = layer.self_attn, layer.mlp
                self.layers.append({
                    "attn_norm": layer.input_layernorm.weight.detach().contiguous(),
                    "w_qkv": torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0).contiguous(),
                    "w_o": a.o_proj.weight.detach().contiguous(),
                    "mlp_norm": layer.post_attention_layernorm.weight.detach().contiguous(),
                    "w_gate_up": _packed_gate_up(m.gate_proj.weight, m.up_proj.weight),
                    "w_down": m.down_proj.weight.detach().contiguous(),
                })
            self.embed = core.embed_tokens.weight.detach().contiguous()
            self.final_norm = core.norm.weight.detach().contiguous()
            self.lm_head = model.lm_head.weight.detach().contiguous()
            rot = core.rotary_emb
            inv_freq = rot.inv_freq.detach().float().cpu()
            scaling = float(getattr(rot, "attention_scaling", 1.0))
            self.max_positions = max(int(getattr(cfg, "max_position_embeddings", 0) or 0), MIN_POSITIONS)
            pos = torch.arange(self.max_positions, dtype=torch.float32)
            freqs = (inv_freq[:, None] @ pos[None, :]).t()   # one fp32 product per entry, as HF forms it
            self.rope_cos = (freqs.cos() * scaling).to(device).contiguous()
            self.rope_sin = (freqs.sin() * scaling).to(device).contiguous()

        self._c_layers = (_ffi.LayerWeights * self.n_layers)()
        for i, L in enumerate(self.layers):
            self._c_layers[i] = _ffi.LayerWeights(ptr(L["attn_norm"]), ptr(L["w_qkv"]), ptr(L["w_o"]), ptr(L["mlp_norm"]),
                                                  ptr(L["w_gate_up"]), ptr(L["w_down"]))
        self._c_weights = _ffi.ModelWeights(ptr(self.embed), ptr(self.final_norm), ptr(self.lm_head),
                                            ptr(self.rope_cos), ptr(self.rope_sin),
                                            ctypes.cast(self._c_layers, ctypes.POINTER(_ffi.LayerWeights)))
        self._c_config = _ffi.ModelConfig(self.n_layers, self.hidden, self.n_heads, self.n_kv_heads, self.head_dim,
                                          self.intermediate, self.vocab, self.eps,
                                          _ffi.BF16 if dtype == torch.bfloat16 else _ffi.F32, self.max_positions)
        handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            raise_for(lib().specb200_model_create(ctypes.byref(self._c_config), ctypes.byref(self._c_weights),
                                                  ctypes.byref(handle)), "specb200_model_create")
        self.handle = handle

    def __del__(self) -> None:
        h = getattr(self, "handle", None)
        if h is not None and _ffi._lib is not None:
            _ffi._lib.specb200_model_destroy(h)

    # ------------------------------------------------------------------ device-level call
    def launches(self, b: int, t: int) -> int:
        """Kernel launches of one forward call of B rows x T tokens."""
        return lib().specb200_forward_launches(self.handle, b, t)

    def schedule(self, b: int, t: int) -> str:
        """The schedule a forward call of B rows x T tokens runs: "gemv" (decode steps of at
        most 4 token rows: a kernel per linear with the norms folded in) or "layers" (a kernel
        per op)."""
        code = lib().specb200_forward_schedule(self.handle, b, t)
        return {3: "gemv"}.get(code, "layers")

    def workspace_bytes(self, b: int, t: int, max_kv_len: int) -> int:
        return lib().specb200_forward_workspace_bytes(self.handle, b, t, max_kv_len)

    def forward_device(self, cache, ids: torch.Tensor, n_new: torch.Tensor, past: torch.Tensor,
                       table: torch.Tensor, max_kv_len: int, last_only: bool, logits: torch.Tensor,
                       status: torch.Tensor, workspace: torch.Tensor | None = None,
                       trace: torch.Tensor | None = None) -> None:
        """Launch the forward on device-resident inputs (no host synchronisation).
        ids [B, T] int32, n_new/past [B] int32, table [B, W] int32, logits fp32 out."""
        b, t = ids.shape
        if cache.k.dtype != self.dtype or cache.k.device != self.device:
            raise ValueError(f"KV pool is {cache.k.dtype} on {cache.k.device}; the model is {self.dtype} on {self.device}")
        if workspace is None:
            workspace = Workspace.get("forward", self.workspace_bytes(b, t, max_kv_len), self.device)
        batch = _ffi.Batch(b, t, ptr(ids), ptr(n_new), ptr(past), ptr(table), table.shape[1], cache.block_size,
                           cache.num_slots, ptr(cache.k), ptr(cache.v), int(last_only), ptr(logits), int(max_kv_len),
                           ptr(status), ptr(trace))
        raise_for(lib().specb200_forward(self.handle, ctypes.byref(batch), ptr(workspace), workspace.numel(),
                                         stream_ptr(self.device)), "specb200_forward")

    # ------------------------------------------------------------------ reference-shaped call
    def forward(self, cache, seq_ids: list[int], input_ids: torch.Tensor, n_new: list[int],
                last_only: bool = False) -> torch.Tensor:
        """lm/forward.py:21-68: run right-padded input_ids [B, T] through the model, appending
        to each sequence's cache; fp32 logits [B, T, V] (or [B, V] with last_only)."""
        dev = self.device
        b, t = input_ids.shape
        past = cache.reserve(seq_ids, n_new)
        max_kv = max(p + n for p, n in zip(past, n_new))
        ids = input_ids.to(dev, torch.int32).contiguous()
        n_new_t = torch.tensor(n_new, dtype=torch.int32).to(dev)
        past_t = torch.tensor(past, dtype=torch.int32).to(dev)
        table = cache.device_tables(seq_ids)
        logits = torch.empty((b, self.vocab) if last_only else (b, t, self.vocab), dtype=torch.float32, device=dev)
        status = Workspace.get("status_fwd", 4, dev)[:4].view(torch.int32)
        self.forward_device(cache, ids, n_new_t, past_t, table, max_kv, last_only, logits, status)
        _ffi.check_status(status, "forward")
        return logits


# Packed engines by model, held weakly so a model can be deep-copied or dropped freely.
_ENGINES: "weakref.WeakKeyDictionary[torch.nn.Module, Engine]" = weakref.WeakKeyDictionary()


def engine_for(model: torch.nn.Module) -> Engine:
    """The model's packed engine, built on first use and rebuilt if the model moved devices
    or changed dtype (weights are assumed fixed after packing, as for inference)."""
    eng = _ENGINES.get(model)
    w = model.model.embed_tokens.weight
    if eng is None or eng.device != w.device or eng.dtype != w.dtype or eng.n_layers != len(model.model.layers):
        eng = Engine(model)
        _ENGINES[model] = eng
    return eng
