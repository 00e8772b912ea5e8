"""Device-resident speculative rounds (filled in with the fused CUDA-graph path)."""
from __future__ import annotations


def fused_path_available(drafter, verify_fn, accept_fn) -> bool:
    return False
