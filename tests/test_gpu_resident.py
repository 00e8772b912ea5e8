"""The resident decode kernel (one cooperative launch per decode step of a draft-class model)
on the GPU, at the full 135M draft architecture (30 layers):

- logits of 1- and 2-token steps of one, two and four sequences against the bf16 oracle, and
  the keys and values those steps wrote into the paged pool against the oracle's cache;
- identical results for identical calls (the packets' launch epochs never let one launch read
  another's data);
- the bounded waits: with a wait limit of a few thousand cycles every wait for another CTA's
  packets gives up, the call reports SPECB200_ERR_TIMEOUT through its status word, and the
  next call with the default limit computes exactly what an undisturbed call computes.
"""
from __future__ import annotations

import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import forward as ofw

sys.path.insert(0, str(GOLDEN))
from recipes import SMOL_135M, llama  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def draft():
    model = llama(SMOL_135M, seed=1, dtype=torch.bfloat16)
    return model, ofw.weights_from_model(model), model.to(DEV)


def _cache(model, blocks: int = 256):
    from cache.kv import KVCache

    return KVCache.for_model(model.config, num_blocks=blocks, block_size=16, dtype=torch.bfloat16, device=DEV)


def test_resident_draft_matches_oracle(draft):
    from lm.forward import forward
    from specb200.engine import engine_for

    _, w, model = draft
    eng = engine_for(model)
    assert eng.schedule(1, 1) == "resident" and eng.schedule(4, 1) == "resident" and eng.schedule(2, 2) == "resident"
    assert eng.launches(1, 1) == 1
    prec = ofw.Precision("bf16")
    cache, ocache = _cache(model), ofw.Cache(w, 256, 16, prec)
    lens = (300, 263, 97, 40)
    for s, n in enumerate(lens):
        cache.add(s)
        ocache.add(s)
        p = torch.randint(0, 49152, (1, n), generator=torch.Generator().manual_seed(70 + s)).numpy()
        forward(model, cache, [s], torch.from_numpy(p), [n], last_only=True)
        ofw.forward(w, ocache, [s], p, [n], prec, last_only=True)
    steps = [([0], [[11]], [1]), ([0, 1], [[12], [13]], [1, 1]), ([0, 1], [[14, 15], [16, 0]], [2, 1]),
             ([1], [[17, 18]], [2]), ([0, 1, 2, 3], [[19], [20], [21], [22]], [1, 1, 1, 1])]
    for seqs, ids, n_new in steps:
        past = [cache.length(s) for s in seqs]
        got = forward(model, cache, seqs, torch.tensor(ids), n_new).float().cpu().numpy()
        want = ofw.forward(w, ocache, seqs, np.array(ids), n_new, prec)
        for b, n in enumerate(n_new):
            g, o = got[b, :n], want[b, :n]
            scale = np.abs(o).max()
            assert np.abs(g - o).max() <= 2e-2 * scale + 1e-3, (seqs, b, np.abs(g - o).max(), scale)
            top2 = np.sort(o, axis=-1)[:, -2:]
            agree = g.argmax(-1) == o.argmax(-1)
            assert np.all(agree | (top2[:, 1] - top2[:, 0] < 2e-2 * scale)), (seqs, b)
        # the keys and values the step wrote, layer by layer, against the oracle's cache
        for b, (s, n) in enumerate(zip(seqs, n_new)):
            slots = cache.tables[s].slots(past[b], past[b] + n, cache.block_size).tolist()
            oslots = list(ocache.tables[s].slots(past[b], past[b] + n, 16))
            for pool, opool in ((cache.k, ocache.k), (cache.v, ocache.v)):
                e = pool[:, torch.tensor(slots)].float().cpu().numpy()
                o = opool[:, oslots]
                # layer 0's entries depend on the step's own tokens only: within one bf16
                # grid step of the oracle. Deeper layers also carry bf16 roundings of every
                # earlier layer, made in another summation order (they drift by a few grid
                # steps over 30 layers); a wrong position, rotation or slot is off by O(1).
                for layer in range(o.shape[0]):
                    d = np.abs(e[layer] - o[layer]).max()
                    bound = (2 ** -7 if layer == 0 else 4e-2) * max(1.0, np.abs(o[layer]).max())
                    assert d <= bound, (s, layer, d)


def test_resident_repeated_calls_are_identical(draft):
    from lm.forward import forward

    _, _, model = draft
    outs = []
    for _ in range(3):
        cache = _cache(model)
        cache.add(0)
        p = torch.randint(0, 49152, (1, 200), generator=torch.Generator().manual_seed(5))
        forward(model, cache, [0], p, [200], last_only=True)
        outs.append([forward(model, cache, [0], torch.tensor([[t]]), [1], last_only=True).cpu() for t in (3, 4, 5)])
    for other in outs[1:]:
        for a, b in zip(outs[0], other):
            assert torch.equal(a, b)


def test_resident_wait_limit_times_out_and_recovers(draft):
    """A wait limit of 2000 cycles (about 1 us) is shorter than any hand-off between CTAs, so
    the call's waits give up: the status word reports a timeout (raised as RuntimeError by the
    wrapper) and no kernel is left running. Restoring the default, the same step on the same
    cache (rolled back) gives the undisturbed result bit for bit."""
    from lm.forward import forward
    from specb200 import _ffi

    _, _, model = draft
    lib = _ffi.lib()
    p = torch.randint(0, 49152, (1, 150), generator=torch.Generator().manual_seed(9))
    ref_cache = _cache(model)
    ref_cache.add(0)
    forward(model, ref_cache, [0], p, [150], last_only=True)
    want = forward(model, ref_cache, [0], torch.tensor([[77]]), [1], last_only=True).cpu()

    cache = _cache(model)
    cache.add(0)
    forward(model, cache, [0], p, [150], last_only=True)
    prev = lib.specb200_set_wait_limit(2000)
    try:
        with pytest.raises(RuntimeError, match="timeout"):
            forward(model, cache, [0], torch.tensor([[77]]), [1], last_only=True)
    finally:
        lib.specb200_set_wait_limit(prev)
    torch.cuda.synchronize()
    cache.truncate(0, 150)
    got = forward(model, cache, [0], torch.tensor([[77]]), [1], last_only=True).cpu()
    assert torch.equal(got, want)
