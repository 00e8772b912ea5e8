"""Oracle: n-gram prompt lookup (spec/ngram.py:32-45 of the reference).

`lookup` calls the C restatement in ngram.c (built by oracle/build.py into oracle/_build/);
`lookup_py` is the same scan in pure Python, used for small cases and to cross-check the C.
"""
from __future__ import annotations

import ctypes

import numpy as np

from oracle.build import build_ngram


def lookup_py(context: list[int], k: int, max_n: int) -> list[int]:
    for n in range(min(max_n, len(context) - 1), 0, -1):
        suffix = context[len(context) - n:]
        for start in range(len(context) - n - 1, -1, -1):
            if context[start:start + n] != suffix:
                continue
            src = context[start + n:]
            out: list[int] = []
            for i in range(k):
                out.append(src[i] if i < len(src) else out[i - len(src)])
            return out
    return [context[-1]] * k


_lib = None


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build_ngram()))
        lib.oracle_ngram_batch.restype = ctypes.c_int
        lib.oracle_ngram_batch.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_void_p]
        _lib = lib
    return _lib


def lookup_batch(contexts: list[list[int]], k: int, max_n: int) -> np.ndarray:
    width = max(len(c) for c in contexts)
    ctx = np.zeros((len(contexts), width), dtype=np.int32)
    for i, c in enumerate(contexts):
        ctx[i, : len(c)] = c
    lens = np.array([len(c) for c in contexts], dtype=np.int32)
    out = np.zeros((len(contexts), k), dtype=np.int64)
    rc = _load().oracle_ngram_batch(ctx.ctypes.data, width, lens.ctypes.data, len(contexts), k, max_n, out.ctypes.data)
    if rc != 0:
        raise IndexError("oracle lookup: empty context")
    return out


def lookup(context: list[int], k: int, max_n: int) -> list[int]:
    return lookup_batch([context], k, max_n)[0].tolist()
