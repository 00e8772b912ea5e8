"""ctypes binding of libspecb200.so (the C ABI declared in include/specb200.h).

This module is the only place that touches the shared library. It loads it from this
package directory (built in-tree by specb200.build), declares every prototype, and turns
the C status codes into the exceptions the reference raises for the same conditions:
ValueError for a drafted token with zero draft probability (spec/accept.py:67-68),
IndexError for out-of-range ids, NotImplementedError for unsupported shapes
(lm/forward.py:14-18), RuntimeError otherwise. There is no CPU fallback: without the
library or without a CUDA device every entry point raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libspecb200.so"

OK, ERR_ARG, ERR_RANGE, ERR_ZERO_Q, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_WORKSPACE = range(8)
F32, BF16 = 0, 1
ACCEPT_LOGITS, ACCEPT_Q_ONEHOT, ACCEPT_DECIDE_ONLY, ACCEPT_Q_STEP_MAJOR = 1, 2, 4, 8

c_int, c_float, c_size_t, c_void_p, c_int64 = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int64


class ModelConfig(ctypes.Structure):
    _fields_ = [("n_layers", c_int), ("hidden", c_int), ("n_heads", c_int), ("n_kv_heads", c_int),
                ("head_dim", c_int), ("intermediate", c_int), ("vocab", c_int), ("rms_eps", c_float),
                ("dtype", c_int), ("max_positions", c_int)]


class LayerWeights(ctypes.Structure):
    _fields_ = [("attn_norm", c_void_p), ("w_qkv", c_void_p), ("w_o", c_void_p), ("mlp_norm", c_void_p),
                ("w_gate_up", c_void_p), ("w_down", c_void_p)]


class ModelWeights(ctypes.Structure):
    _fields_ = [("embed", c_void_p), ("final_norm", c_void_p), ("lm_head", c_void_p), ("rope_cos", c_void_p),
                ("rope_sin", c_void_p), ("layers", ctypes.POINTER(LayerWeights))]


class Batch(ctypes.Structure):
    _fields_ = [("B", c_int), ("T", c_int), ("input_ids", c_void_p), ("n_new", c_void_p), ("past_len", c_void_p),
                ("block_table", c_void_p), ("table_stride", c_int), ("block_size", c_int), ("num_slots", c_int),
                ("k_pool", c_void_p), ("v_pool", c_void_p), ("last_only", c_int), ("logits", c_void_p),
                ("max_kv_len", c_int), ("status", c_void_p), ("trace", c_void_p)]


# name -> (restype, argtypes)
PROTOTYPES: dict[str, tuple] = {
    "specb200_version": (c_int, []),
    "specb200_last_error": (ctypes.c_char_p, []),
    "specb200_wait_probe": (c_int, [c_void_p, c_void_p, c_void_p]),
    "specb200_accept_workspace_bytes": (c_size_t, [c_int, c_int]),
    "specb200_accept": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float,
                                c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "specb200_probabilities": (c_int, [c_void_p, c_int, c_int, c_float, c_void_p, c_void_p]),
    "specb200_accept_noalloc_max_rows": (c_size_t, []),
    "specb200_accept_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                        c_float, c_void_p, c_void_p, c_void_p, c_void_p]),
    "specb200_ngram": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "specb200_commit_tokens": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                       c_int, c_void_p]),
    "specb200_verify_ids": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                    c_void_p, c_void_p]),
    "specb200_scatter_tokens": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "specb200_logit_noise": (c_int, [c_void_p, c_int, c_int, c_int64, c_void_p, c_void_p, c_void_p, ctypes.c_uint64,
                                     c_float, c_void_p]),
    "specb200_model_create": (c_int, [ctypes.POINTER(ModelConfig), ctypes.POINTER(ModelWeights),
                                      ctypes.POINTER(c_void_p)]),
    "specb200_model_destroy": (c_int, [c_void_p]),
    "specb200_forward_workspace_bytes": (c_size_t, [c_void_p, c_int, c_int, c_int]),
    "specb200_forward_schedule": (c_int, [c_void_p, c_int, c_int]),
    "specb200_forward_launches": (c_int, [c_void_p, c_int, c_int]),
    "specb200_forward": (c_int, [c_void_p, ctypes.POINTER(Batch), c_void_p, c_size_t, c_void_p]),
    "specb200_rmsnorm": (c_int, [c_int, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p]),
    "specb200_linear_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "specb200_linear": (c_int, [c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_size_t,
                                c_void_p, c_void_p]),
    "specb200_attention_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "specb200_attention": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                   c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p, c_size_t,
                                   c_void_p, c_void_p]),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library, with prototypes declared. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m specb200.build` "
                               "(the engine has no CPU fallback)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class ZeroDraftMass(ValueError):
    pass


def raise_for(code: int, where: str) -> None:
    if code == OK:
        return
    msg = f"{where}: {lib().specb200_last_error().decode(errors='replace')}"
    if code == ERR_ZERO_Q:
        raise ZeroDraftMass("a drafted token has zero draft probability; q is not what it was sampled from")
    if code == ERR_RANGE:
        raise IndexError(msg or f"{where}: index out of range")
    if code == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if code == ERR_ARG:
        raise ValueError(msg)
    raise RuntimeError(f"{msg} (status {code})")


def check_status(status: torch.Tensor, where: str) -> None:
    """Reads device status words (synchronises with their stream) and raises on the first
    error found."""
    words = status.reshape(-1)
    bad = words[words != 0]
    code = int(bad[0].item()) if bad.numel() else 0
    if code == ERR_ZERO_Q:
        raise ZeroDraftMass("a drafted token has zero draft probability; q is not what it was sampled from")
    if code == ERR_RANGE:
        raise IndexError(f"{where}: a token id, position or pool slot is out of range")
    if code == ERR_TIMEOUT:
        raise RuntimeError(f"{where}: a device-side wait gave up (timeout)")
    if code == ERR_WORKSPACE:
        raise RuntimeError(f"{where}: the workspace held stale state (it must be zero-filled before its first use)")
    if code != OK:
        raise RuntimeError(f"{where}: device status {code}")


def require_cuda(t: torch.Tensor, where: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(f"{where}: the B200 engine runs on CUDA tensors only (got {t.device})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class Workspace:
    """Zero-filled, grow-only scratch buffers on the device, one per purpose and device.
    The kernels leave counters at zero, so a buffer is zeroed only when (re)allocated."""

    _buffers: dict[tuple[str, int], torch.Tensor] = {}

    @classmethod
    def get(cls, name: str, nbytes: int, device: torch.device) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        key = (name, idx)
        buf = cls._buffers.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 16)
            if buf is not None:
                size = max(size, 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
            cls._buffers[key] = buf
        return buf
