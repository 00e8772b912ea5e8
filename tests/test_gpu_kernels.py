"""Kernel-level parity on the GPU, through the C ABI: fused accept-reject and sampling, n-gram
lookup, RMSNorm, the tcgen05 / FFMA linear layers and paged attention, each against the
oracle, the reference's golden vectors and known-answer tests, or a plain fp32 torch
computation of the same op (stated tolerance per test)."""
from __future__ import annotations

from fractions import Fraction

import numpy as np
import pytest
import torch

from oracle import accept as oacc
from oracle import forward as ofw
from oracle import ngram as ong

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ops():
    from specb200 import ops

    return ops


# ---------------------------------------------------------------- accept-reject (K8/K10)
@pytest.mark.parametrize("name", ["t1", "t07", "t0"])
def test_accept_logits_mode_matches_reference(golden_accept, name):
    g = golden_accept
    T = float(g[f"{name}_temperature"])
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(DEV)  # noqa: E731
    n, nxt = _ops().accept(t(g[f"{name}_p_logits"]), t(g[f"{name}_q_logits"]), t(g[f"{name}_draft"]),
                           t(g[f"{name}_u_accept"]), t(g[f"{name}_u_residual"]), logits=True, temperature=T)
    assert n.cpu().numpy().tolist() == g[f"{name}_n"].tolist()
    assert nxt.cpu().numpy().tolist() == g[f"{name}_next"].tolist()


def test_accept_onehot_mode_matches_reference(golden_accept):
    g = golden_accept
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(DEV)  # noqa: E731
    n, nxt = _ops().accept(t(g["hot_p_logits"]), None, t(g["hot_draft"]), t(g["hot_u_accept"]),
                           t(g["hot_u_residual"]), logits=True, temperature=1.0, q_onehot=True)
    assert n.cpu().tolist() == g["hot_n"].tolist() and nxt.cpu().tolist() == g["hot_next"].tolist()


def test_inverse_cdf_matches_reference(golden_accept):
    from spec.accept import sample_inverse_cdf

    g = golden_accept
    got = sample_inverse_cdf(torch.from_numpy(g["cdf_probs"]).to(DEV), torch.from_numpy(g["cdf_u"]).to(DEV))
    assert got.cpu().tolist() == g["cdf_token"].tolist()


# The reference's tests/test_accept_toy.py, through the drop-in accept_reject.
P = [Fraction(4, 10), Fraction(3, 10), Fraction(2, 10), Fraction(1, 10), Fraction(0)]
Q = [Fraction(1, 10), Fraction(2, 10), Fraction(3, 10), Fraction(1, 10), Fraction(3, 10)]
ACCEPT = [Fraction(1), Fraction(1), Fraction(2, 3), Fraction(1), Fraction(0)]


def _t(xs):
    return torch.tensor([float(x) for x in xs], dtype=torch.float64)


def test_scripted_uniforms():
    from spec.accept import accept_reject

    p = _t(P).expand(1, 2, 5)
    q = _t(Q).expand(1, 1, 5)
    d = torch.tensor([[2]])
    run = lambda ua, ur: accept_reject(p, q, d, u_accept=torch.tensor([[ua]], dtype=torch.float64),  # noqa: E731
                                       u_residual=torch.tensor([ur], dtype=torch.float64))
    a = run(0.6, 0.5)
    assert a.n_accepted.item() == 1 and a.next_token.item() == 1
    r = run(0.7, 0.8)
    assert r.n_accepted.item() == 0 and r.next_token.item() == 1
    assert run(0.7, 0.5).next_token.item() == 0


def test_zero_target_mass_is_never_emitted():
    from spec.accept import accept_reject

    v = accept_reject(_t(P).expand(1000, 2, 5), _t(Q).expand(1000, 1, 5), torch.full((1000, 1), 4),
                      generator=torch.Generator().manual_seed(0))
    assert v.n_accepted.sum().item() == 0 and set(v.next_token.tolist()) <= {0, 1}


def test_coupled_stream_reproduces_target_exactly():
    """120-point grid of both uniforms (tests/test_accept_toy.py:54-76): every acceptance and
    inverse-CDF interval holds a whole number of grid points, so the output distribution is
    exactly P as fractions."""
    from spec.accept import accept_reject

    n = 120
    grid = (torch.arange(n, dtype=torch.float64) + 0.5) / n
    ua = grid.repeat_interleave(n).unsqueeze(-1)
    ur = grid.repeat(n)
    p = _t(P).expand(n * n, 2, 5)
    q = _t(Q).expand(n * n, 1, 5)
    emitted = [Fraction(0)] * 5
    for y in range(5):
        if Q[y] == 0:
            continue
        d = torch.full((n * n, 1), y)
        v = accept_reject(p, q, d, u_accept=ua, u_residual=ur)
        first = torch.where(v.n_accepted == 1, d[:, 0], v.next_token)
        assert Fraction(int(v.n_accepted.sum()), n * n) == ACCEPT[y]
        for x, c in enumerate(torch.bincount(first, minlength=5).tolist()):
            emitted[x] += Q[y] * Fraction(c, n * n)
    assert emitted == P


def test_greedy_reduces_to_argmax_verification():
    from spec.accept import accept_reject

    p = torch.nn.functional.one_hot(torch.tensor([[3, 1, 4]]), 5).double()
    d = torch.tensor([[3, 2]])
    v = accept_reject(p, torch.nn.functional.one_hot(d, 5).double(), d, generator=torch.Generator().manual_seed(0))
    assert v.n_accepted.item() == 1 and v.next_token.item() == 1
    d2 = torch.tensor([[3, 1]])
    v = accept_reject(p, torch.nn.functional.one_hot(d2, 5).double(), d2, generator=torch.Generator().manual_seed(0))
    assert v.n_accepted.item() == 2 and v.next_token.item() == 4


def test_inverse_cdf_skips_zero_mass():
    from spec.accept import sample_inverse_cdf

    probs = torch.tensor([[0.0, 0.5, 0.0, 0.5, 0.0]], dtype=torch.float64)
    for u, want in [(0.0, 1), (0.49, 1), (0.5, 3), (0.999, 3)]:
        assert sample_inverse_cdf(probs, torch.tensor([u], dtype=torch.float64)).item() == want


def test_zero_draft_mass_raises():
    from spec.accept import accept_reject

    q = torch.tensor([[[0.5, 0.5, 0.0]]])
    with pytest.raises(ValueError, match="zero draft probability"):
        accept_reject(torch.full((1, 2, 3), 1 / 3), q, torch.tensor([[2]]), generator=torch.Generator().manual_seed(0))


def test_distribution_matches_target_and_catches_broken_residual():
    """A condensed tests/test_accept_distribution.py: 100k seeded rounds at V=32, k=4; the
    first emitted token's distribution fits p, and resampling p on rejection does not."""
    from scipy.stats import chisquare

    from spec.accept import accept_reject

    N, V, K = 100_000, 32, 4
    torch.manual_seed(0)
    d = torch.distributions.Dirichlet(torch.ones(V, dtype=torch.float64))
    p, q = d.sample(), d.sample()
    gen = torch.Generator().manual_seed(2)
    draft = torch.multinomial(q, N * K, replacement=True, generator=gen).view(N, K)
    pe, qe = p.expand(N, K + 1, V), q.expand(N, K, V)
    v = accept_reject(pe, qe, draft, generator=gen)
    first = torch.where(v.n_accepted >= 1, draft[:, 0], v.next_token)
    counts = torch.bincount(first, minlength=V).double()
    assert chisquare(counts.numpy(), (p * N).numpy()).pvalue > 1e-3
    gen = torch.Generator().manual_seed(2)
    draft = torch.multinomial(q, N * K, replacement=True, generator=gen).view(N, K)
    bad = accept_reject(pe, qe, draft, generator=gen, residual=lambda pp, qq: pp)
    first = torch.where(bad.n_accepted >= 1, draft[:, 0], bad.next_token)
    counts = torch.bincount(first, minlength=V).double()
    assert chisquare(counts.numpy(), (p * N).numpy()).pvalue < 1e-3


@pytest.mark.parametrize("temperature", [1.0, 0.0])
def test_accept_config3_size_matches_oracle(temperature):
    """BASELINE config 3 shape (B=64, k=4, V=49152; target logits N(0, 3^2), draft = target +
    N(0, 1)): decisions identical to the oracle except where |p_x - u q_x| < 1e-5, tokens
    identical except where u * total sits within 1e-5 (relative) of a CDF boundary."""
    B, K, V = 64, 4, 49152
    g = torch.Generator().manual_seed(3)
    pl = torch.randn(B, K + 1, V, generator=g) * 3.0
    ql = pl[:, :K] + torch.randn(B, K, V, generator=g)
    qp = oacc.probabilities(ql.numpy(), temperature)
    if temperature > 0:
        draft = torch.multinomial(torch.from_numpy(qp).reshape(-1, V), 1, generator=g).reshape(B, K)
    else:
        draft = torch.from_numpy(qp.argmax(-1))
    ua, ur = torch.rand(B, K, generator=g), torch.rand(B, generator=g)
    n, nxt = _ops().accept(pl.to(DEV), ql.to(DEV), draft.to(DEV), ua.to(DEV), ur.to(DEV), logits=True,
                           temperature=temperature)
    on, onxt = oacc.accept_reject_logits(pl.numpy(), ql.numpy(), draft.numpy(), ua.numpy(), ur.numpy(), temperature)
    n, nxt = n.cpu().numpy(), nxt.cpu().numpy()
    pp = oacc.probabilities(pl.numpy(), temperature)
    mismatched_rows = np.nonzero((n != on) | (nxt != onxt))[0]
    for b in mismatched_rows:
        m = min(n[b], on[b])
        px = pp[b, m, draft[b, m]] if m < K else 1.0
        qx = qp[b, m, draft[b, m]] if m < K else 0.0
        if n[b] != on[b]:  # a different decision: only where u q_x sits within 1e-5 of p_x
            assert m < K and abs(px - ua[b, m].item() * qx) < 1e-5, (b, n[b], on[b])
            continue
        # same decision, different sample: u * total must sit within 1e-5 (relative) of the
        # oracle's CDF at the boundary the two tokens straddle (the residual of row n, or p
        # itself at the bonus row)
        qrow = qp[b, m] if m < K else np.zeros(V, dtype=np.float32)
        r = oacc.residual_distribution(pp[b, m][None], qrow[None])[0]
        cdf = np.cumsum(r.astype(np.float64)).astype(np.float32)
        target = np.float32(ur[b].item()) * cdf[-1]
        lo, hi = sorted((int(nxt[b]), int(onxt[b])))
        assert abs(float(cdf[lo]) - float(target)) <= 1e-5 * float(cdf[-1]), (b, lo, cdf[lo], target)
        assert abs(float(cdf[hi - 1]) - float(target)) <= 1e-5 * float(cdf[-1]), (b, hi, cdf[hi - 1], target)
    assert len(mismatched_rows) <= 2


def test_accept_calls_of_different_shapes_share_one_workspace():
    """One zero-filled workspace serves accept calls of any (B, k) and mode in turn (the
    engine's round alternates k = 0 samplers with the (B, k) accept on one buffer): every call
    matches the oracle's decisions and greedy tokens, and leaves the whole workspace zero."""
    from specb200 import _ffi

    lib = _ffi.lib()
    nbytes = max(lib.specb200_accept_workspace_bytes(b, k) for b, k in ((7, 4), (1, 0), (3, 2), (64, 4)))
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    g = torch.Generator().manual_seed(91)
    for B, K, V, temp in ((7, 4, 4096, 0.0), (1, 0, 49152, 1.0), (3, 2, 1000, 0.7), (64, 4, 4096, 1.0),
                          (1, 0, 49152, 0.0), (7, 4, 4096, 1.0), (3, 2, 1000, 0.0)):
        pl = torch.randn(B, K + 1, V, generator=g) * 2.0
        ql = pl[:, :K] + torch.randn(B, K, V, generator=g)
        qp = oacc.probabilities(ql.numpy(), temp)
        draft = (torch.from_numpy(qp.argmax(-1)) if temp == 0 else
                 torch.multinomial(torch.from_numpy(qp).reshape(-1, V), 1, generator=g).reshape(B, K)) if K else \
            torch.zeros(B, 1, dtype=torch.int64)
        ua, ur = torch.rand(B, max(K, 1), generator=g), torch.rand(B, generator=g)
        d = {n: t.to(DEV).contiguous() for n, t in (("p", pl), ("q", ql), ("d", draft), ("ua", ua), ("ur", ur))}
        n_acc = torch.empty(B, dtype=torch.int64, device=DEV)
        nxt = torch.empty(B, dtype=torch.int64, device=DEV)
        rc = lib.specb200_accept(d["p"].data_ptr(), d["q"].data_ptr() if K else None, d["d"].data_ptr(),
                                 d["ua"].data_ptr(), d["ur"].data_ptr(), B, K, V, _ffi.ACCEPT_LOGITS, temp,
                                 n_acc.data_ptr(), nxt.data_ptr(), status.data_ptr(), ws.data_ptr(), ws.numel(),
                                 torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert int(torch.count_nonzero(ws).item()) == 0, (B, K, V, temp)
        on, onxt = oacc.accept_reject_logits(pl.numpy(), ql.numpy(), draft.numpy()[:, :K], ua.numpy()[:, :K],
                                             ur.numpy(), temp)
        got_n, got_t = n_acc.cpu().numpy(), nxt.cpu().numpy()
        if temp == 0:
            assert np.array_equal(got_n, on) and np.array_equal(got_t, onxt), (B, K, V)
        else:  # sampled: decisions and tokens agree except at the 1e-5 boundaries (config-3 test)
            assert (got_n != on).sum() + (got_t != onxt).sum() <= 1, (B, K, V)


# ---------------------------------------------------------------- n-gram (K9)
def test_ngram_matches_reference_golden(golden_ngram):
    from spec.ngram import lookup

    for case in golden_ngram:
        assert lookup(case["context"], case["k"], case["max_n"]) == case["draft"], case


def test_ngram_batch_long_contexts_match_oracle():
    rng = np.random.default_rng(0)
    contexts = []
    for i in range(32):
        n = int(rng.integers(1, 8448))
        vocab = [3, 50, 49152][i % 3]
        contexts.append(rng.integers(0, vocab, n).tolist())
    from spec.ngram import contexts_tensor

    ctx, lens = contexts_tensor(contexts, torch.device(DEV))
    for k, max_n in ((4, 3), (6, 3), (8, 8), (1, 1)):
        got = _ops().ngram(ctx, lens, k, max_n).cpu().numpy()
        assert (got == ong.lookup_batch(contexts, k, max_n)).all()


def test_ngram_reference_kats():
    from spec.ngram import lookup

    assert lookup([1, 2, 3, 4, 1, 2], k=2, max_n=3) == [3, 4]
    assert lookup([1, 2, 3, 1, 2], k=5, max_n=2) == [3, 1, 2, 3, 1]
    ctx = [7, 8, 9, 1, 8, 5, 7, 8]
    assert lookup(ctx, k=1, max_n=2) == [9] and lookup(ctx, k=1, max_n=1) == [5]
    assert lookup([1, 4, 2, 4, 3, 4], k=1, max_n=1) == [3]
    assert lookup([1, 2, 3], k=3, max_n=3) == [3, 3, 3]


# ---------------------------------------------------------------- RMSNorm (K2)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H", [576, 2048, 8200, 100])
def test_rmsnorm_matches_hf_formula(dtype, H):
    """Vectorised rows held in registers (576, 2048), the scalar path past the register budget
    (8200 elements) and for rows that are not whole 16-byte chunks (100 bf16 elements)."""
    x = (torch.randn(7, H, generator=torch.Generator().manual_seed(1)) * 2).to(DEV, dtype)
    w = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(2))).to(DEV, dtype)
    xf = x.float()
    ref = w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).to(dtype)
    got = _ops().rmsnorm(x, w, 1e-5)
    tol = 0 if dtype == torch.float32 else 1e-2
    assert (got.float() - ref.float()).abs().max().item() <= max(tol, 2e-6)


# ---------------------------------------------------------------- linear layers (K3/K5/K6/K7)
@pytest.mark.parametrize("m,n,k", [(5, 128, 64), (5, 960, 576), (5, 6144, 2048), (16, 2048, 8192), (40, 384, 256),
                                   (1, 49152, 576), (300, 640, 512), (129, 256, 128)])
def test_linear_bf16_tcgen05_matches_fp32_torch(m, n, k):
    """bf16 inputs, fp32 accumulation in TMEM: within 1e-3 relative of a fp32 torch matmul of
    the same bf16 values (summation order only)."""
    g = torch.Generator().manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, generator=g).to(DEV, torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.05).to(DEV, torch.bfloat16)
    ref = x.float() @ w.float().t()
    got = _ops().linear(x, w, out_f32=True)
    err = (got - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item() + 1e-4, err


@pytest.mark.parametrize("m,n,k", [(5, 128, 64), (3, 960, 576), (40, 384, 256)])
def test_linear_fp32_matches_torch(m, n, k):
    g = torch.Generator().manual_seed(n + k)
    x = torch.randn(m, k, generator=g).to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.05).to(DEV)
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = x @ w.t()
    got = _ops().linear(x, w, out_f32=True)
    assert (got - ref).abs().max().item() <= 1e-4


# ---------------------------------------------------------------- paged attention (K4)
@pytest.mark.parametrize("dtype,hq,hkv,d,T,bs,long_past", [
    (torch.float32, 4, 2, 16, 5, 4, 700), (torch.bfloat16, 32, 32, 64, 5, 16, 700),
    (torch.bfloat16, 9, 3, 64, 2, 16, 700), (torch.float32, 4, 4, 32, 40, 3, 700),
    (torch.bfloat16, 9, 3, 64, 1, 16, 700), (torch.bfloat16, 9, 3, 64, 5, 16, 700),
    (torch.bfloat16, 12, 3, 64, 4, 32, 700), (torch.bfloat16, 32, 4, 64, 3, 16, 700),
    (torch.bfloat16, 9, 3, 64, 1, 16, 4500), (torch.bfloat16, 4, 2, 64, 4, 1, 130),
    (torch.bfloat16, 9, 3, 64, 1, 32, 8448), (torch.bfloat16, 32, 32, 64, 7, 32, 8448),
    (torch.bfloat16, 32, 32, 64, 5, 32, 8448), (torch.bfloat16, 9, 3, 64, 40, 16, 700),
    (torch.bfloat16, 4, 2, 64, 130, 1, 90), (torch.bfloat16, 32, 32, 64, 200, 32, 300),
    (torch.bfloat16, 64, 64, 64, 5, 16, 700), (torch.bfloat16, 128, 64, 64, 3, 16, 700)])
def test_attention_matches_dense_reference(dtype, hq, hkv, d, T, bs, long_past):
    """Paged attention over shuffled blocks vs the reference's mask (lm/forward.py:44-49) on
    a dense fp32 copy: rows of lengths 1 .. long_past incl. a padded row. bf16 shapes with at
    most 16 query rows per KV head (T x G) run the cluster kernel (1, 6, 8, 15 and 16 rows
    here; C = 3 .. 8 CTAs per cluster, block size 1 included) or, when the keys exceed one
    cluster (4500 cached, and config 5's 8448 at block 32 for the 135M and 1.7B head
    layouts, T = 1, 5 and 7), the tensor-core split items; bf16 prefill shapes (120, 260 and
    200 query rows per KV head, block sizes 16, 1 and 32) the tensor-core prefill kernel;
    decode shapes with many (sequence, KV head) pairs (3 x 64 pairs with 5 and 6 query rows
    each, as a B = 64 verify's 64 x 32) the tensor-core split items; 24 rows (32 / 4 heads,
    T = 3) and the fp32 cases run the fp32 items."""
    g = torch.Generator().manual_seed(hq + T)
    lens_past = [0, 37, long_past]
    n_new = [T, max(1, T - 2), T]
    B = len(lens_past)
    total = [p + n for p, n in zip(lens_past, n_new)]
    blocks_per = [-(-t // bs) for t in total]
    num_blocks = sum(blocks_per) + 5
    perm = torch.randperm(num_blocks, generator=g).tolist()
    width = max(blocks_per)
    table = torch.zeros(B, width, dtype=torch.int32)
    it = iter(perm)
    for b in range(B):
        for j in range(blocks_per[b]):
            table[b, j] = next(it)
    kp = torch.randn(num_blocks * bs, hkv, d, generator=g).to(DEV, dtype)
    vp = torch.randn(num_blocks * bs, hkv, d, generator=g).to(DEV, dtype)
    q = torch.randn(B, T, hq, d, generator=g).to(DEV, dtype)
    scale = d ** -0.5
    out = _ops().attention(q, kp, vp, table.to(DEV), bs, torch.tensor(lens_past, dtype=torch.int32, device=DEV),
                           torch.tensor(n_new, dtype=torch.int32, device=DEV), scale, max(total))
    for b in range(B):
        slots = torch.tensor([table[b, j // bs].item() * bs + j % bs for j in range(total[b])])
        kk = kp[slots].float().repeat_interleave(hq // hkv, dim=1)
        vv = vp[slots].float().repeat_interleave(hq // hkv, dim=1)
        for t in range(T):
            pos = lens_past[b] + t
            allowed = torch.arange(total[b], device=DEV) <= pos
            sc = torch.einsum("hd,shd->hs", q[b, t].float(), kk) * scale
            sc = sc.masked_fill(~allowed[None], float("-inf"))
            ref = torch.einsum("hs,shd->hd", sc.softmax(-1), vv)
            tol = 2e-5 if dtype == torch.float32 else 1.5e-2
            assert (out[b, t].float() - ref).abs().max().item() <= tol, (b, t)


# ---------------------------------------------------------------- bounded device waits
def test_bounded_wait_gives_up_and_context_stays_usable():
    """A kernel waits, with the bounded helper every pipeline uses for its mbarrier waits, on a
    phase that nothing completes: the wait gives up after its spin limit (about 2 s at the boost
    clock), the status word reads SPECB200_ERR_TIMEOUT and the abort flag was raised; the
    context then runs a real kernel (greedy accept-reject) correctly."""
    import time

    from specb200 import _ffi
    from specb200._ffi import lib, ptr

    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    gave_up = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert lib().specb200_wait_probe(ptr(status), ptr(gave_up), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert status.item() == _ffi.ERR_TIMEOUT and gave_up.item() == 1, (status.item(), gave_up.item())
    assert 0.2 < waited < 30.0, waited
    g = torch.Generator(device=DEV).manual_seed(5)
    pl = torch.randn(3, 3, 64, generator=g, device=DEV)
    draft = pl[:, :2].argmax(-1)
    n, nxt = _ops().accept(pl, None, draft, torch.zeros(3, 2, device=DEV), torch.zeros(3, device=DEV), logits=True,
                           temperature=0.0, q_onehot=True)
    assert n.tolist() == [2, 2, 2] and nxt.tolist() == pl[:, 2].argmax(-1).tolist()
