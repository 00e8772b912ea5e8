"""The allocation-free accept entry point (specb200_accept_noalloc), through the C ABI.

Callers that cannot allocate device memory (a runtime that reserves all HBM up front, or an
operator interface that passes only inputs and outputs) use this variant: its scratch is a
fixed device array inside the library instead of a caller workspace. It must give exactly the
results of specb200_accept on the same inputs, call after call, although the array keeps each
call's leftovers. This file is collected last on purpose, and runs alone as well.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(seed: int, B: int, k: int, V: int, temperature: float):
    """Config-3 style logits; drafts drawn from q as a drafter would (argmax at T = 0)."""
    g = torch.Generator().manual_seed(seed)
    pl = torch.randn(B, k + 1, V, generator=g) * 3.0
    ql = pl[:, :k] + torch.randn(B, k, V, generator=g)
    if k == 0:
        draft = torch.zeros(B, 0, dtype=torch.int64)
    elif temperature == 0.0:
        draft = ql.argmax(-1)
    else:
        draft = torch.multinomial(torch.softmax(ql / temperature, -1).reshape(-1, V), 1, generator=g).reshape(B, k)
    ua, ur = torch.rand(B, k, generator=g), torch.rand(B, generator=g)
    return [t.to(DEV).contiguous() for t in (pl, ql, draft, ua, ur)]


def _with_workspace(lib, pl, ql, draft, ua, ur, flags, temperature):
    B, k1, V = pl.shape
    n = torch.full((B,), -1, dtype=torch.int64, device=DEV)
    nxt = torch.full((B,), -1, dtype=torch.int64, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ws = torch.zeros(lib.specb200_accept_workspace_bytes(B, k1 - 1), dtype=torch.uint8, device=DEV)
    rc = lib.specb200_accept(pl.data_ptr(), ql.data_ptr(), draft.data_ptr(), ua.data_ptr(), ur.data_ptr(), B, k1 - 1, V,
                             flags, temperature, n.data_ptr(), nxt.data_ptr(), status.data_ptr(), ws.data_ptr(),
                             ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    return n, nxt, status


def _no_alloc(lib, pl, ql, draft, ua, ur, flags, temperature):
    B, k1, V = pl.shape
    n = torch.full((B,), -1, dtype=torch.int64, device=DEV)
    nxt = torch.full((B,), -1, dtype=torch.int64, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib.specb200_accept_noalloc(pl.data_ptr(), ql.data_ptr(), draft.data_ptr(), ua.data_ptr(), ur.data_ptr(), B,
                                     k1 - 1, V, flags, temperature, n.data_ptr(), nxt.data_ptr(), status.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.specb200_last_error()
    return n, nxt, status


@pytest.mark.parametrize("temperature", [1.0, 0.0])
def test_no_alloc_matches_workspace_entry_point_on_consecutive_calls(temperature):
    """Calls in a row with different inputs and batch sizes (each starts on the previous one's
    leftover tickets and statistics): decisions and tokens identical to the workspace entry
    point, as integers."""
    from specb200 import _ffi

    lib = _ffi.lib()
    flags = _ffi.ACCEPT_LOGITS
    # Config-3 sizes take one CTA per row; the few-row shapes (the draft sampler's B = 1, k = 0
    # and a small verify batch) split each row over column chunks whose partial statistics and
    # row tickets also live in the shared array.
    for seed, B, k, V in ((11, 64, 4, 49152), (12, 37, 4, 5000), (13, 1, 0, 49152), (14, 4, 4, 49152),
                          (15, 1, 0, 49152)):
        args = _inputs(seed, B, k, V, temperature)
        n_ref, nxt_ref, st_ref = _with_workspace(lib, *args, flags, temperature)
        n, nxt, st = _no_alloc(lib, *args, flags, temperature)
        torch.cuda.synchronize()
        assert int(st.item()) == 0 and int(st_ref.item()) == 0
        assert torch.equal(n, n_ref)
        assert torch.equal(nxt, nxt_ref)
        assert int(n.min()) >= 0 and int(nxt.min()) >= 0


def test_no_alloc_rejects_batches_beyond_its_scratch():
    from specb200 import _ffi

    lib = _ffi.lib()
    max_rows = lib.specb200_accept_noalloc_max_rows()
    assert max_rows == 512
    one = torch.zeros(1, device=DEV)
    rc = lib.specb200_accept_noalloc(one.data_ptr(), None, None, None, one.data_ptr(), max_rows + 1, 0, 1, 0, 1.0,
                                     one.data_ptr(), one.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    assert rc == _ffi.ERR_ARG
    assert b"512" in lib.specb200_last_error()
