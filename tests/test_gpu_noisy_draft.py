"""The noisy-copy drafter of BASELINE config 2's second variant on the GPU (the target itself
as the draft, with seeded N(0, sigma^2) noise on its final logits; the reference has no such
drafter, so the CPU oracle's restatement is the checker).

- specb200_logit_noise against oracle.noise: the same Philox words, normals to fp32 rounding,
  rows with no new tokens untouched.
- spec.loop.generate with NoisyDraft on the tiny fp32 model against the oracle's generate
  with its NoisyDraft: identical outputs and SpecStats, greedy and sampled, on the fused round
  and on the composable path.
- Exactness: greedy output with the noisy drafter equals plain decoding, at an acceptance
  strictly between 0 and 1.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import tiny_fp32
from oracle import forward as ofw
from oracle import loop as oloop
from oracle import noise as onoise

pytestmark = pytest.mark.gpu
DEV = "cuda"
SIGMA = 0.4


@pytest.fixture(scope="module")
def tiny():
    return tiny_fp32().to(DEV)


def _cache(model, blocks: int = 2048, block_size: int = 4):
    from cache.kv import KVCache

    return KVCache.for_model(model.config, num_blocks=blocks, block_size=block_size, dtype=model.dtype, device=DEV)


def test_logit_noise_kernel_matches_oracle():
    from specb200 import _ffi

    lib = _ffi.lib()
    B, V, seed, sigma = 5, 49152, 0x1234_5678_9ABC, 0.75
    logits = torch.randn(B, V, generator=torch.Generator().manual_seed(1))
    past = torch.tensor([0, 17, 300, 4000, 9], dtype=torch.int32)
    n_new = torch.tensor([1, 2, 0, 5, 1], dtype=torch.int32)
    rows = torch.tensor([3, 0, 1, 7, 2], dtype=torch.int32)
    got = logits.to(DEV)
    d_past, d_new, d_rows = past.to(DEV), n_new.to(DEV), rows.to(DEV)  # alive until the kernel has run
    rc = lib.specb200_logit_noise(got.data_ptr(), B, V, V, d_past.data_ptr(), d_new.data_ptr(), d_rows.data_ptr(),
                                  seed, sigma, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    want = logits.numpy().copy()
    live = [b for b in range(B) if n_new[b] > 0]
    want[live] = onoise.add_noise(want[live], seed, sigma, rows[live].tolist(), (past + n_new)[live].tolist())
    assert np.array_equal(got[2], logits.numpy()[2])  # n_new = 0: untouched
    assert np.abs(got - want).max() <= 1e-5 * sigma * 8


def _oracle_generate(model, prompts, max_new, k, temperature, seed_gen):
    w = ofw.weights_from_model(model)
    prec = ofw.Precision("f32")
    drafter = oloop.NoisyDraft(w, prec, num_blocks=2048, block_size=4, sigma=SIGMA, seed=11)
    gen = torch.Generator().manual_seed(seed_gen)
    return oloop.generate(w, prec, drafter, prompts, max_new, k, temperature=temperature, generator=gen,
                          num_blocks=2048, block_size=4)


@pytest.mark.parametrize("path", ["fused", "composable"])
@pytest.mark.parametrize("temperature", [0.0, 1.0])
def test_noisy_draft_generate_matches_oracle(tiny, path, temperature, monkeypatch):
    from conftest import random_prompts
    from spec.draft import NoisyDraft
    from spec.loop import generate

    if path == "composable":
        monkeypatch.setattr("specb200.rounds.fused_path_available", lambda *a: False)
    prompts = random_prompts(6, 256, seed=21)
    cpu_model = tiny_fp32()
    want_out, want = _oracle_generate(cpu_model, prompts, 20, 4, temperature, 5)
    out, st = generate(tiny, _cache(tiny), NoisyDraft(tiny, _cache(tiny), sigma=SIGMA, seed=11), prompts, 20, k=4,
                       temperature=temperature, generator=torch.Generator().manual_seed(5))
    assert out == want_out
    for key in ("rounds", "drafted", "accepted", "attempts", "accepts", "emitted_per_round", "drafted_per_round"):
        assert getattr(st, key) == want[key], key
    assert 0 < st.accepted < st.drafted  # neither a copy nor a useless draft at this sigma


def test_noisy_draft_greedy_equals_plain_decode(tiny):
    from baselines import cached_autoregressive
    from conftest import random_prompts
    from spec.draft import NoisyDraft
    from spec.loop import generate

    prompts = random_prompts(8, 256, seed=22)
    out, st = generate(tiny, _cache(tiny), NoisyDraft(tiny, _cache(tiny), sigma=SIGMA, seed=3), prompts, 24, k=4)
    for p, o in zip(prompts, out):
        assert o == cached_autoregressive.generate(tiny, _cache(tiny), p, 24)
    assert 0 < st.accepted < st.drafted
