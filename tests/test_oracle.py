"""The oracle pinned against the reference's own outputs (tests/golden/, made by
tests/golden/make_golden.py). CPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import tiny_fp32
from oracle import accept as oacc
from oracle import forward as ofw
from oracle import loop as oloop
from oracle import ngram as ong
from oracle import paged as opg


@pytest.mark.parametrize("name", ["t1", "t07", "t0"])
def test_accept_matches_reference(golden_accept, name):
    g = golden_accept
    T = float(g[f"{name}_temperature"])
    n, nxt = oacc.accept_reject_logits(g[f"{name}_p_logits"], g[f"{name}_q_logits"], g[f"{name}_draft"],
                                       g[f"{name}_u_accept"], g[f"{name}_u_residual"], T)
    assert (n == g[f"{name}_n"]).all()
    assert (nxt == g[f"{name}_next"]).all()


def test_onehot_draft_matches_reference(golden_accept):
    g = golden_accept
    n, nxt = oacc.accept_reject_logits(g["hot_p_logits"], None, g["hot_draft"], g["hot_u_accept"],
                                       g["hot_u_residual"], 1.0)
    assert (n == g["hot_n"]).all() and (nxt == g["hot_next"]).all()


def test_inverse_cdf_matches_reference(golden_accept):
    g = golden_accept
    assert (oacc.sample_inverse_cdf(g["cdf_probs"], g["cdf_u"]) == g["cdf_token"]).all()


def test_accept_toy_fractions():
    """The hand-computed case of the reference's tests/test_accept_toy.py:7-42."""
    P = np.array([0.4, 0.3, 0.2, 0.1, 0.0], dtype=np.float32)
    Q = np.array([0.1, 0.2, 0.3, 0.1, 0.3], dtype=np.float32)
    r = oacc.residual_distribution(P, Q)
    assert np.allclose(r, [0.75, 0.25, 0, 0, 0], atol=1e-7)
    p = np.broadcast_to(P, (1, 2, 5)).copy()
    q = np.broadcast_to(Q, (1, 1, 5)).copy()
    d = np.array([[2]])
    run = lambda ua, ur: oacc.accept_reject(p, q, d, np.array([[ua]], np.float32), np.array([ur], np.float32))  # noqa: E731
    assert run(0.6, 0.5)[0][0] == 1 and run(0.6, 0.5)[1][0] == 1
    assert run(0.7, 0.8)[0][0] == 0 and run(0.7, 0.8)[1][0] == 1
    assert run(0.7, 0.5)[1][0] == 0


def test_ngram_c_and_python_match_reference(golden_ngram):
    for case in golden_ngram:
        assert ong.lookup(case["context"], case["k"], case["max_n"]) == case["draft"], case
        assert ong.lookup_py(case["context"], case["k"], case["max_n"]) == case["draft"], case


def test_paged_walk_matches_reference(golden_paged):
    bs = golden_paged["block_size"]
    alloc = opg.Allocator(golden_paged["num_blocks"])
    tables: dict[int, opg.Table] = {}
    for op, s, arg, snapshot in golden_paged["log"]:
        if op == "add":
            tables[s] = opg.Table()
        elif op == "append":
            tables[s].grow_to(tables[s].length + arg, alloc, bs)
        elif op == "append_oob":
            with pytest.raises(opg.OutOfBlocks):
                tables[s].grow_to(tables[s].length + arg, alloc, bs)
        elif op == "truncate":
            tables[s].shrink_to(arg, alloc, bs)
        else:
            tables[s].shrink_to(0, alloc, bs)
            del tables[s]
        assert {str(k): [t.blocks, t.length] for k, t in tables.items()} == snapshot


def _forward_rounds(golden, bs, prec):
    w = ofw.weights_from_model(tiny_fp32().to(torch.float64))
    cache = ofw.Cache(w, 256, bs, prec)
    for s in range(3):
        cache.add(s)
    out = []
    for r in range(4):
        out.append((ofw.forward(w, cache, [0, 1, 2], golden[f"bs{bs}_r{r}_ids"], list(golden[f"bs{bs}_r{r}_n_new"]),
                                prec), golden[f"bs{bs}_r{r}_logits"], golden[f"bs{bs}_r{r}_n_new"]))
    cache.truncate(0, cache.length(0) - 2)
    out.append((ofw.forward(w, cache, [0], golden[f"bs{bs}_trunc_ids"], [3], prec), golden[f"bs{bs}_trunc_logits"],
                np.array([3])))
    return out


@pytest.mark.parametrize("bs", [1, 4])
def test_forward_f64_matches_reference(golden_forward, bs):
    """The fp64 oracle forward reproduces the reference's cached forward to 1e-10, the
    reference's own equivalence bar (tests/test_cache_equivalence.py:14)."""
    for got, want, n_new in _forward_rounds(golden_forward, bs, ofw.Precision("f64")):
        for b, n in enumerate(n_new):
            assert np.abs(got[b, :n] - want[b, :n]).max() <= 1e-10


def test_tiny_weights_match_fixture(golden_forward):
    sd = tiny_fp32().state_dict()
    for k, v in sd.items():
        assert np.array_equal(v.numpy(), golden_forward["w_" + k]), k


@pytest.mark.parametrize("name", ["ngram_k1", "ngram_k4", "draft_k1", "draft_k4"])
def test_generate_matches_reference(golden_generate, name):
    g = golden_generate
    tiny = tiny_fp32().to(torch.float64)
    w = ofw.weights_from_model(tiny)
    prec = ofw.Precision("f64")
    k = int(name[-1])
    if name.startswith("ngram"):
        drafter = oloop.NGramDraft(256)
    else:
        wd = dict(w)
        wd["layers"] = w["layers"][:1]
        drafter = oloop.ModelDraft(wd, prec, 4096, 4)
    prompts = g["prompts"] + g["repetitive"]
    out, stats = oloop.generate(w, prec, drafter, prompts, g["max_new"], k, num_blocks=4096, block_size=4)
    want = g[name]
    assert out == want["outputs"]
    for key in ("rounds", "drafted", "accepted", "attempts", "accepts", "emitted_per_round", "drafted_per_round"):
        assert stats[key] == want[key], key


def test_plain_decode_matches_reference(golden_generate):
    g = golden_generate
    w = ofw.weights_from_model(tiny_fp32().to(torch.float64))
    prec = ofw.Precision("f64")
    for p, want in zip(g["prompts"][:8] + g["repetitive"], g["plain"][:8] + g["plain"][-1:]):
        assert oloop.generate_plain(w, prec, p, g["max_new"], block_size=4) == want


def test_philox_matches_known_answers():
    """The noise oracle's Philox4x32-10 against the known-answer vectors published with the
    generator (Salmon et al., SC 2011, Random123 kat_vectors: zero, all-ones and pi-digit
    counters and keys)."""
    from oracle.noise import philox4x32_10

    cases = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
             ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
             ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
              (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for ctr, key, want in cases:
        got = philox4x32_10(*ctr, *key)
        assert tuple(int(x) for x in got) == want


def test_logit_noise_is_standard_normal_and_keyed():
    """The noise is N(0, 1) per element (moments and a normality test over 2 x 49152 draws),
    depends on every key field, and adds sigma * z to the logits row by row."""
    from scipy.stats import normaltest

    from oracle.noise import add_noise, normals

    z = np.concatenate([normals(7, 0, 512, 49152), normals(7, 1, 513, 49152)])
    assert abs(z.mean()) < 0.02 and abs(z.std() - 1.0) < 0.02
    assert normaltest(z).pvalue > 1e-3
    base = normals(7, 0, 512, 64)
    for other in (normals(8, 0, 512, 64), normals(7, 1, 512, 64), normals(7, 0, 513, 64)):
        assert not np.allclose(base, other)
    logits = np.ones((2, 64), dtype=np.float32)
    out = add_noise(logits, 7, 0.5, [0, 1], [512, 513])
    np.testing.assert_allclose(out[0], 1 + 0.5 * base, rtol=1e-6)
    np.testing.assert_allclose(out[1], 1 + 0.5 * normals(7, 1, 513, 64), rtol=1e-6)
