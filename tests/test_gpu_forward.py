"""Forward and round parity on the GPU: the engine's cached forward against the reference's
fp64 logits (golden) and the bf16 oracle, and spec.loop.generate / plain decoding against the
reference's outputs and statistics on the tiny model, plus the reference's rollback and
bonus-token tests."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch
from transformers import LlamaConfig, LlamaForCausalLM

from conftest import early_exit, random_prompts, tiny_fp32
from oracle import forward as ofw

pytestmark = pytest.mark.gpu
DEV = "cuda"


def new_cache(model, block_size: int = 4, num_blocks: int = 4096):
    from cache.kv import KVCache

    return KVCache.for_model(model.config, num_blocks=num_blocks, block_size=block_size, dtype=model.dtype, device=DEV)


@pytest.fixture(scope="module")
def tiny():
    return tiny_fp32().to(DEV)


# ---------------------------------------------------------------- forward
@pytest.mark.parametrize("bs", [1, 4])
def test_forward_fp32_matches_reference_fp64(tiny, golden_forward, bs):
    """Mixed-length padded batches, multi-token appends and truncate-then-append: the fp32
    engine is within 2e-5 of the reference's fp64 logits on identical weights."""
    from lm.forward import forward

    g = golden_forward
    cache = new_cache(tiny, block_size=bs, num_blocks=256)
    for s in range(3):
        cache.add(s)
    for r in range(4):
        n_new = [int(x) for x in g[f"bs{bs}_r{r}_n_new"]]
        got = forward(tiny, cache, [0, 1, 2], torch.from_numpy(g[f"bs{bs}_r{r}_ids"]), n_new).cpu().numpy()
        want = g[f"bs{bs}_r{r}_logits"]
        for b, n in enumerate(n_new):
            assert np.abs(got[b, :n] - want[b, :n]).max() <= 2e-5, (r, b)
    cache.truncate(0, cache.length(0) - 2)
    got = forward(tiny, cache, [0], torch.from_numpy(g[f"bs{bs}_trunc_ids"]), [3]).cpu().numpy()
    assert np.abs(got - g[f"bs{bs}_trunc_logits"]).max() <= 2e-5


def _bf16_model(hidden, layers, heads, kv, inter, vocab, seed, theta=10000.0):
    cfg = LlamaConfig(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=kv, max_position_embeddings=8192,
                      rope_parameters={"rope_type": "default", "rope_theta": theta}, rms_norm_eps=1e-5,
                      tie_word_embeddings=True, attn_implementation="sdpa")
    torch.manual_seed(seed)
    return LlamaForCausalLM(cfg).to(torch.bfloat16).eval()


@pytest.mark.parametrize("dims", [(128, 2, 2, 1, 256, 512), (576, 2, 9, 3, 1536, 49152), (2048, 2, 32, 32, 8192, 49152)])
def test_forward_bf16_matches_oracle(dims):
    """bf16 engine (tcgen05 GEMMs) vs the bf16 oracle over a prefill and a (k+1)-token verify:
    logits within rtol 2e-2 of the largest logit, argmax agreeing except at near ties."""
    from lm.forward import forward

    model = _bf16_model(*dims, seed=11, theta=130000.0)
    w = ofw.weights_from_model(model)
    prec = ofw.Precision("bf16")
    model = model.to(DEV)
    cache = new_cache(model, block_size=16)
    ocache = ofw.Cache(w, 4096, 16, prec)
    prompts = [torch.randint(0, dims[-1], (n,), generator=torch.Generator().manual_seed(n)).tolist() for n in (40, 17)]
    for s in range(2):
        cache.add(s)
        ocache.add(s)
    width = 40
    ids = np.array([p + [0] * (width - len(p)) for p in prompts])
    steps = [(ids, [40, 17]), (np.array([[1, 2, 3, 4, 5], [6, 7, 8, 9, 10]]), [5, 5])]
    for ids_np, n_new in steps:
        got = forward(model, cache, [0, 1], torch.from_numpy(ids_np), n_new).float().cpu().numpy()
        want = ofw.forward(w, ocache, [0, 1], ids_np, n_new, prec)
        for b, n in enumerate(n_new):
            g, o = got[b, :n], want[b, :n]
            scale = np.abs(o).max()
            assert np.abs(g - o).max() <= 2e-2 * scale + 1e-3, (b, np.abs(g - o).max(), scale)
            top2 = np.sort(o, axis=-1)[:, -2:]
            gap = top2[:, 1] - top2[:, 0]
            agree = g.argmax(-1) == o.argmax(-1)
            assert np.all(agree | (gap < 2e-2 * scale)), (b, gap[~agree])


# ---------------------------------------------------------------- generate
@pytest.fixture(params=["fused", "composable"])
def path(request, monkeypatch):
    """Run generate() through the CUDA-graph round (engine drafters) or through the
    module-by-module path that custom drafters and patched verify/accept_reject take."""
    if request.param == "composable":
        monkeypatch.setattr("specb200.rounds.fused_path_available", lambda *a: False)
    return request.param


@pytest.mark.parametrize("name", ["ngram_k1", "ngram_k4", "draft_k1", "draft_k4"])
def test_generate_matches_reference(tiny, golden_generate, name, path):
    """Greedy spec.loop.generate on the fp32 engine reproduces the reference's fp64 outputs
    and every SpecStats counter."""
    from spec.draft import ModelDraft
    from spec.loop import generate
    from spec.ngram import NGramDraft

    g = golden_generate
    k = int(name[-1])
    drafter = NGramDraft(256) if name.startswith("ngram") else ModelDraft(early_exit(tiny), None)
    if isinstance(drafter, ModelDraft):
        drafter.cache = new_cache(drafter.model)
    out, st = generate(tiny, new_cache(tiny), drafter, g["prompts"] + g["repetitive"], g["max_new"], k=k)
    want = g[name]
    assert out == want["outputs"]
    for key in ("rounds", "drafted", "accepted", "attempts", "accepts", "emitted_per_round", "drafted_per_round"):
        assert getattr(st, key) == want[key], key


def test_sampled_generate_matches_reference(tiny, golden_generate, path):
    """Temperature 1 with a seeded generator: the uniforms are drawn in the reference's order,
    so draft samples, accept decisions and residual samples reproduce its output."""
    from spec.draft import ModelDraft
    from spec.loop import generate

    g = golden_generate
    d = early_exit(tiny)
    out, st = generate(tiny, new_cache(tiny), ModelDraft(d, new_cache(d)), g["prompts"][:6], 16, k=3,
                       temperature=1.0, generator=torch.Generator().manual_seed(5))
    assert out == g["sampled_draft_k3"]["outputs"]
    assert (st.accepted, st.drafted) == (g["sampled_draft_k3"]["accepted"], g["sampled_draft_k3"]["drafted"])


def test_fused_path_is_taken_for_engine_drafters(tiny, monkeypatch):
    from spec.loop import generate
    from spec.ngram import NGramDraft
    from specb200 import rounds

    calls = []
    real = rounds.generate_fused
    monkeypatch.setattr(rounds, "generate_fused", lambda *a, **kw: calls.append(1) or real(*a, **kw))
    out, _ = generate(tiny, new_cache(tiny), NGramDraft(256), [[1, 2, 3, 1, 2]], 8, k=4)
    assert calls == [1] and len(out[0]) == 8


def test_fused_round_keeps_the_allocator_caches(tiny, monkeypatch):
    """Capturing the round's graph must not return cached device or pinned host blocks to the
    driver: re-allocating them for every request stalled requests for hundreds of ms."""
    from spec.loop import generate
    from spec.ngram import NGramDraft

    calls = []
    dev_empty, host_empty = torch.cuda.empty_cache, torch._C._host_emptyCache
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: calls.append("device") or dev_empty())
    monkeypatch.setattr(torch._C, "_host_emptyCache", lambda: calls.append("host") or host_empty())
    for _ in range(2):
        out, _ = generate(tiny, new_cache(tiny), NGramDraft(256), [[4, 8, 15, 16, 23, 42, 4, 8]], 10, k=3)
        assert len(out[0]) == 10
    assert calls == []


def test_plain_decode_matches_reference(tiny, golden_generate):
    from baselines import cached_autoregressive

    g = golden_generate
    for p, want in zip(g["prompts"] + g["repetitive"], g["plain"]):
        assert cached_autoregressive.generate(tiny, new_cache(tiny), p, g["max_new"]) == want


def test_batched_plain_decode_matches_one_at_a_time(tiny, golden_generate):
    from baselines import cached_autoregressive

    g = golden_generate
    cache = new_cache(tiny, block_size=16, num_blocks=128)
    prompts = g["prompts"]
    for i in range(0, len(prompts), 8):
        assert cached_autoregressive.generate_batch(tiny, cache, prompts[i:i + 8], g["max_new"]) == g["plain"][i:i + 8]
    assert cache.allocator.num_used == 0 and not cache.tables


def test_eos_stops_mid_window(tiny, golden_generate, path):
    """With eos set to a token the reference emits partway through a request, the request
    ends right after its first occurrence, inside a verify window (the reference's
    tests/test_greedy_identity.py:76-82)."""
    from spec.draft import ModelDraft
    from spec.loop import generate

    g = golden_generate
    want = g["draft_k4"]["outputs"][0]
    eos = want[5]
    d = early_exit(tiny)
    out, _ = generate(tiny, new_cache(tiny), ModelDraft(d, new_cache(d)), [g["prompts"][0]], g["max_new"], k=4,
                      eos_id=eos)
    assert out[0] == want[: want.index(eos) + 1]


def test_uniform_draft_is_still_exact(tiny, golden_generate):
    """A custom drafter that proposes uniform noise (the composable path) accepts almost
    nothing, and the output is still the target's greedy continuation."""
    from spec.draft import UniformDraft
    from spec.loop import generate

    g = golden_generate
    out, st = generate(tiny, new_cache(tiny), UniformDraft(tiny.config.vocab_size), g["prompts"], g["max_new"], k=4,
                       generator=torch.Generator().manual_seed(0))
    assert out == g["plain"][: len(g["prompts"])]
    assert st.accepted / st.drafted < 0.05


def test_batched_plain_decode_drops_a_row_at_eos(tiny):
    """Batched plain decoding retires a row at its eos and finishes the others, as one-at-a-time
    decoding does (the reference's tests/test_batch_size.py:31-37)."""
    from baselines import cached_autoregressive

    prompts = [[5, 6, 7], list(range(30, 60))]
    full = [cached_autoregressive.generate(tiny, new_cache(tiny), p, 12) for p in prompts]
    eos = full[0][3]
    want = [cached_autoregressive.generate(tiny, new_cache(tiny), p, 12, eos_id=eos) for p in prompts]
    assert len(want[0]) <= 4
    assert cached_autoregressive.generate_batch(tiny, new_cache(tiny), prompts, 12, eos_id=eos) == want


class ScriptedDraft:
    """Proposes the target's own continuation for the first j positions, then a wrong token
    (the reference's tests/test_rollback.py:13-34)."""

    def __init__(self, reference, prompt_len, j, vocab):
        self.reference, self.prompt_len, self.j, self.vocab = reference, prompt_len, j, vocab

    def prefill(self, seq_ids, prompts):
        pass

    def propose(self, seq_ids, contexts, k, temperature, generator):
        done = len(contexts[0]) - self.prompt_len
        right = self.reference[done:done + k] + [0] * k
        draft = [right[i] if i < self.j else (right[i] + 1) % self.vocab for i in range(k)]
        tokens = torch.tensor([draft])
        return tokens, torch.nn.functional.one_hot(tokens, self.vocab).float()

    def rollback(self, seq_id, keep):
        pass

    def release(self, seq_id):
        pass


@pytest.mark.parametrize("j", range(5))
def test_exactly_j_accepted_every_round(tiny, j):
    from baselines import cached_autoregressive
    from spec.loop import generate

    prompt = random_prompts(1, 256, seed=3)[0]
    want = cached_autoregressive.generate(tiny, new_cache(tiny), prompt, 30 + 5)
    out, st = generate(tiny, new_cache(tiny), ScriptedDraft(want, len(prompt), j, 256), [prompt], 30, k=4)
    assert out[0] == want[:30]
    assert st.accepts[:j] == st.attempts[:j] and all(a == 0 for a in st.accepts[j:])
    assert all(e == j + 1 for e in st.emitted_per_round[:-1])


@pytest.mark.parametrize(("k", "max_new"), [(1, 20), (4, 21), (4, 23), (7, 30)])
def test_full_acceptance_emits_k_plus_one(tiny, k, max_new):
    from baselines import cached_autoregressive
    from spec.draft import ModelDraft
    from spec.loop import generate

    prompt = random_prompts(1, 256, seed=5)[0]
    want = cached_autoregressive.generate(tiny, new_cache(tiny), prompt, max_new)
    out, st = generate(tiny, new_cache(tiny), ModelDraft(tiny, new_cache(tiny)), [prompt], max_new, k=k)
    assert out[0] == want
    assert st.rounds == math.ceil((max_new - 1) / (k + 1))
    assert all(e == k + 1 for e in st.emitted_per_round[:-1])


def test_sampled_copy_draft_never_rejects(tiny):
    from spec.draft import ModelDraft
    from spec.loop import generate

    prompts = random_prompts(20, 256, seed=6)
    _, st = generate(tiny, new_cache(tiny), ModelDraft(tiny, new_cache(tiny)), prompts, 20, k=4, temperature=1.0,
                     generator=torch.Generator().manual_seed(0))
    assert st.accepted == st.drafted


def test_verify_invariant_raises(tiny):
    from spec.verify import verify

    cache = new_cache(tiny)
    cache.add(0)
    with pytest.raises(RuntimeError, match="target cache holds"):
        verify(tiny, cache, [0], [[1, 2, 3]], torch.tensor([[4, 5]]), 0.0)


def _gemv_steps(eng, model, prompt_len: int = 300, pad_to: int = 0):
    """Prefill two sequences, then decode-sized calls (at most 4 token rows) of every shape the
    GEMV schedule serves: 1 row x 1 token, 2 rows x 1 token (last rows), 2 rows x 2 tokens with
    a ragged row, 1 row x 3 tokens. With pad_to, every call is right-padded to that many tokens
    per row (padding writes no K/V), which moves it to the per-layer kernels. Returns the real
    rows' logits and the final KV pools."""
    from cache.kv import KVCache

    cache = KVCache.for_model(model.config, num_blocks=96, block_size=16, dtype=torch.bfloat16, device=DEV)
    for s in range(2):
        cache.add(s)
        n = prompt_len - 37 * s
        p = torch.randint(0, model.config.vocab_size, (1, n), generator=torch.Generator().manual_seed(50 + s))
        eng.forward(cache, [s], p, [n], last_only=True)

    def call(seqs, rows, n_new, last_only=False):
        width = max(pad_to, max(len(r) for r in rows))
        ids = torch.tensor([r + [0] * (width - len(r)) for r in rows])
        out = eng.forward(cache, seqs, ids, n_new, last_only=last_only).float().cpu()
        return out if last_only else torch.cat([out[b, :n] for b, n in enumerate(n_new)])

    outs = [call([0], [[11]], [1], True), call([0, 1], [[12], [13]], [1, 1], True),
            call([0, 1], [[14, 15], [16]], [2, 1]), call([1], [[17, 18, 19]], [3])]
    return outs, cache


@pytest.mark.parametrize("dims", [(576, 2, 9, 3, 1536, 49152), (256, 2, 4, 4, 512, 49152),
                                  (128, 2, 4, 2, 256, 512)])
def test_decode_schedules_match_per_layer_kernels(dims):
    """Decode-sized calls (at most 4 token rows) on the GEMV kernels against the same tokens
    padded to 5 per row, which run on the tensor-core per-layer kernels: the 135M draft width, a
    narrow model with the same vocabulary and a head_dim-32 model with a small one (whose LM
    head is a GEMV too); 2 layers each. The schedules sum in different orders, so logits agree
    to bf16 noise (1e-2 of the logit scale, argmax equal except at near ties) and the KV entries
    the calls wrote to one bf16 ulp of their scale."""
    from specb200.engine import Engine

    model = _bf16_model(*dims, seed=8, theta=100000.0).to(DEV)
    eng = Engine(model)
    assert eng.schedule(1, 1) == "gemv" and eng.schedule(2, 2) == "gemv" and eng.schedule(1, 3) == "gemv"
    assert eng.schedule(1, 5) == "layers" and eng.schedule(2, 5) == "layers"
    # prep, 5 per layer, then the LM head: a GEMV with the final norm folded in (small
    # vocabulary) or the final norm and the tensor-core GEMM
    head_launches = 1 if dims[-1] <= 4096 else 2
    assert eng.launches(1, 1) == 1 + head_launches + 5 * 2
    assert eng.launches(1, 5) == 3 + 7 * 2
    (la, ca), (lb, cb) = _gemv_steps(eng, model, pad_to=5), _gemv_steps(eng, model)
    for a, b in zip(la, lb):
        scale = a.abs().max().item()
        assert (a - b).abs().max().item() <= 1e-2 * scale, ((a - b).abs().max().item(), scale)
        top2 = a.topk(2, dim=-1).values
        agree = a.argmax(-1) == b.argmax(-1)
        assert bool((agree | ((top2[..., 0] - top2[..., 1]) < 1e-2 * scale)).all())
    for pa, pb in ((ca.k, cb.k), (ca.v, cb.v)):
        d = (pa.float() - pb.float()).abs().max().item()
        assert d <= 2 ** -7 * pa.float().abs().max().item(), d


@pytest.mark.parametrize("dims", [(576, 2, 9, 3, 1536, 49152), (128, 2, 4, 2, 256, 512)])
def test_decode_schedules_match_oracle(dims):
    """The decode-step GEMV schedule (at the 135M width and at a narrow width) against the bf16
    oracle: after a prefill, 1-token steps of one and of two sequences and a
    3-token step, logits within rtol 2e-2 of the largest logit."""
    from lm.forward import forward
    from specb200.engine import engine_for

    model = _bf16_model(*dims, seed=13, theta=100000.0)
    w = ofw.weights_from_model(model)
    prec = ofw.Precision("bf16")
    model = model.to(DEV)
    assert engine_for(model).schedule(1, 1) == "gemv"
    cache = new_cache(model, block_size=16)
    ocache = ofw.Cache(w, 4096, 16, prec)
    for s in range(2):
        cache.add(s)
        ocache.add(s)
    prompts = [torch.randint(0, dims[-1], (1, n), generator=torch.Generator().manual_seed(n)).numpy() for n in (70, 33)]
    steps = [([0], prompts[0], [70]), ([1], prompts[1], [33]), ([0], np.array([[6]]), [1]),
             ([0, 1], np.array([[7], [8]]), [1, 1]), ([1], np.array([[9, 10, 11]]), [3])]
    for seqs, ids_np, n_new in steps:
        got = forward(model, cache, seqs, torch.from_numpy(ids_np), n_new).float().cpu().numpy()
        want = ofw.forward(w, ocache, seqs, ids_np, n_new, prec)
        for b, n in enumerate(n_new):
            g, o = got[b, :n], want[b, :n]
            scale = np.abs(o).max()
            assert np.abs(g - o).max() <= 2e-2 * scale + 1e-3, (b, np.abs(g - o).max(), scale)


def test_long_prefill_matches_oracle():
    """A 1100-token prefill and a 300-token continuation (tensor-core prefill attention over 18
    and 22 key blocks per query tile; prefill-sized GEMM token tiles) of a 2-layer bf16 model
    with grouped heads, against the bf16 oracle: last-position logits of the prefill and every
    position's logits of the continuation, within rtol 2e-2 of the largest logit."""
    from lm.forward import forward

    model = _bf16_model(256, 2, 8, 2, 512, 4096, seed=17, theta=130000.0)
    w = ofw.weights_from_model(model)
    prec = ofw.Precision("bf16")
    model = model.to(DEV)
    cache = new_cache(model, block_size=16)
    ocache = ofw.Cache(w, 4096, 16, prec)
    cache.add(0)
    ocache.add(0)
    g = torch.Generator().manual_seed(33)
    for n, last in ((1100, True), (300, False)):
        ids = torch.randint(0, 4096, (1, n), generator=g)
        got = forward(model, cache, [0], ids, [n], last_only=last).float().cpu().numpy()
        want = ofw.forward(w, ocache, [0], ids.numpy(), [n], prec, last_only=last)
        scale = np.abs(want).max()
        assert np.abs(got - want).max() <= 2e-2 * scale + 1e-3, (n, np.abs(got - want).max(), scale)
