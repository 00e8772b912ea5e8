"""Generate the golden vectors in tests/golden/ by running the reference implementation.

    python tests/golden/make_golden.py /path/to/speculative-decoder

The reference (beriltatli/speculative-decoder, pure Python + PyTorch) is imported read-only
from the given checkout in this process only; nothing in the engine, the oracle or the GPU
tests reads it at run time. Every fixture is produced by the reference's own functions on
seeded inputs:

  accept.npz      spec/accept.py accept_reject / sample_inverse_cdf and lm/sampling.py
                  probabilities, on fp32 logits with explicit uniforms (sampling and greedy)
  ngram.json      spec/ngram.py lookup on random small-vocabulary contexts
  paged.json      cache/paged.py + cache/kv.py: a seeded random walk of add/append/truncate/
                  free, with the block ids of every table after each operation
  forward.npz     lm/forward.py forward on the tiny fp64 Llama (lm/load.py tiny_model seed 0,
                  whose weights are exact fp32 values): prefill, mixed-length appends,
                  truncate-then-append, at block sizes 1 and 4; weights included
  generate.json   spec/loop.py generate (n-gram and early-exit model drafts, k in {1, 4}) and
                  baselines/cached_autoregressive.py generate on the tiny fp64 model
"""
from __future__ import annotations

import copy
import json
import random
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def main(ref: str) -> None:
    sys.path.insert(0, ref)
    from cache.kv import KVCache
    from cache.paged import OutOfBlocks
    from lm.forward import forward
    from lm.load import tiny_model
    from lm.sampling import probabilities
    from spec.accept import accept_reject, sample_inverse_cdf
    from spec.draft import ModelDraft
    from spec.loop import generate
    from spec.ngram import NGramDraft, lookup
    from baselines import cached_autoregressive

    torch.set_num_threads(4)

    # ---------------------------------------------------------------- accept
    g = torch.Generator().manual_seed(1234)
    B, K, V = 24, 4, 96
    out = {}
    for name, temp in (("t1", 1.0), ("t07", 0.7), ("t0", 0.0)):
        pl = torch.randn(B, K + 1, V, generator=g) * 3.0
        ql = pl[:, :K] + torch.randn(B, K, V, generator=g)
        if temp == 0.0:
            # some rows draft exactly the target's argmax, so the bonus path is covered
            ql[: B // 3] = pl[: B // 3, :K]
        q = probabilities(ql, temp)
        draft = torch.multinomial(q.reshape(-1, V), 1, generator=g).reshape(B, K) if temp > 0 else q.argmax(-1)
        ua = torch.rand(B, K, generator=g)
        ur = torch.rand(B, generator=g)
        p = probabilities(pl, temp)
        v = accept_reject(p, q, draft, u_accept=ua, u_residual=ur)
        out.update({f"{name}_p_logits": pl.numpy(), f"{name}_q_logits": ql.numpy(), f"{name}_draft": draft.numpy(),
                    f"{name}_u_accept": ua.numpy(), f"{name}_u_residual": ur.numpy(),
                    f"{name}_temperature": np.float32(temp), f"{name}_n": v.n_accepted.numpy(),
                    f"{name}_next": v.next_token.numpy()})
    # inverse CDF with zero-mass gaps
    probs = torch.rand(64, V, generator=g)
    probs[probs < 0.5] = 0
    u = torch.rand(64, generator=g)
    out["cdf_probs"] = probs.numpy()
    out["cdf_u"] = u.numpy()
    out["cdf_token"] = sample_inverse_cdf(probs, u).numpy()
    # one-hot draft (n-gram style) at T = 1
    pl = torch.randn(B, K + 1, V, generator=g) * 2.0
    draft = torch.randint(0, V, (B, K), generator=g)
    draft[: B // 2] = pl[: B // 2, :K].argmax(-1)
    q = torch.nn.functional.one_hot(draft, V).float()
    ua, ur = torch.rand(B, K, generator=g), torch.rand(B, generator=g)
    v = accept_reject(probabilities(pl, 1.0), q, draft, u_accept=ua, u_residual=ur)
    out.update({"hot_p_logits": pl.numpy(), "hot_draft": draft.numpy(), "hot_u_accept": ua.numpy(),
                "hot_u_residual": ur.numpy(), "hot_n": v.n_accepted.numpy(), "hot_next": v.next_token.numpy()})
    np.savez_compressed(OUT / "accept.npz", **out)

    # ---------------------------------------------------------------- ngram
    rng = random.Random(7)
    cases = [([1, 2, 3, 4, 1, 2], 2, 3), ([1, 2, 3, 1, 2], 5, 2), ([7, 8, 9, 1, 8, 5, 7, 8], 1, 2),
             ([7, 8, 9, 1, 8, 5, 7, 8], 1, 1), ([1, 4, 2, 4, 3, 4], 1, 1), ([1, 2, 3], 3, 3), ([5], 4, 3),
             ([9, 9], 3, 3), ([1, 1, 1, 1], 6, 3)]
    for _ in range(300):
        n = rng.randint(1, 120)
        vocab = rng.choice([2, 3, 5, 20, 1000])
        ctx = [rng.randrange(vocab) for _ in range(n)]
        cases.append((ctx, rng.choice([1, 2, 4, 6, 8]), rng.choice([1, 2, 3, 4, 8])))
    ngram = [{"context": c, "k": k, "max_n": m, "draft": lookup(c, k, m)} for c, k, m in cases]
    (OUT / "ngram.json").write_text(json.dumps(ngram))

    # ---------------------------------------------------------------- paged random walk
    rng = random.Random(0)
    bs = 3
    cache = KVCache(n_layers=1, n_kv_heads=1, head_dim=8, num_blocks=40, block_size=bs, dtype=torch.float32,
                    device="cpu")
    live, next_id, log = [], 0, []
    for _ in range(600):
        op = rng.random()
        if op < 0.2 or not live:
            cache.add(next_id)
            live.append(next_id)
            step = ["add", next_id, 0]
            next_id += 1
        elif op < 0.6:
            s = rng.choice(live)
            n = rng.randint(1, 7)
            try:
                cache.append([s], [n])
                step = ["append", s, n]
            except OutOfBlocks:
                step = ["append_oob", s, n]
        elif op < 0.85:
            s = rng.choice(live)
            n = rng.randint(0, cache.length(s))
            cache.truncate(s, n)
            step = ["truncate", s, n]
        else:
            s = live.pop(rng.randrange(len(live)))
            cache.free(s)
            step = ["free", s, 0]
        step.append({str(sid): [t.blocks[:], t.length] for sid, t in cache.tables.items()})
        log.append(step)
    (OUT / "paged.json").write_text(json.dumps({"block_size": bs, "num_blocks": 40, "log": log}))

    # ---------------------------------------------------------------- forward (tiny fp64)
    tiny = tiny_model(seed=0, dtype=torch.float64)
    sd = {k: v.numpy().astype(np.float32) for k, v in tiny.state_dict().items()}
    fw = {"w_" + k: v for k, v in sd.items()}
    fw["inv_freq"] = tiny.model.rotary_emb.inv_freq.float().numpy()
    gen = torch.Generator().manual_seed(2)
    for bsz in (1, 4):
        seqs = [torch.randint(0, 256, (n,), generator=gen).tolist() for n in (3, 9, 6)]
        cache = KVCache.for_model(tiny.config, num_blocks=256, block_size=bsz, dtype=torch.float64, device="cpu")
        for s in range(3):
            cache.add(s)
        rounds = [[len(s) for s in seqs], [1, 3, 2], [2, 1, 1], [1, 1, 5]]
        for r, n_new in enumerate(rounds):
            if r > 0:
                for s, n in zip(seqs, n_new):
                    s.extend(torch.randint(0, 256, (n,), generator=gen).tolist())
            chunks = [s[len(s) - n:] for s, n in zip(seqs, n_new)]
            width = max(n_new)
            ids = torch.tensor([c + [0] * (width - len(c)) for c in chunks])
            logits = forward(tiny, cache, [0, 1, 2], ids, n_new)
            fw[f"bs{bsz}_r{r}_ids"] = ids.numpy()
            fw[f"bs{bsz}_r{r}_n_new"] = np.array(n_new)
            fw[f"bs{bsz}_r{r}_logits"] = logits.numpy()
        # truncate then append on sequence 0
        cache.truncate(0, cache.length(0) - 2)
        ids = torch.tensor([[5, 6, 7]])
        logits = forward(tiny, cache, [0], ids, [3])
        fw[f"bs{bsz}_trunc_ids"] = ids.numpy()
        fw[f"bs{bsz}_trunc_logits"] = logits.numpy()
    np.savez_compressed(OUT / "forward.npz", **fw)

    # ---------------------------------------------------------------- generate (tiny fp64)
    def random_prompts(n, vocab, seed, low=3, high=20):
        gg = torch.Generator().manual_seed(seed)
        lengths = torch.randint(low, high, (n,), generator=gg).tolist()
        return [torch.randint(0, vocab, (m,), generator=gg).tolist() for m in lengths]

    def new_cache(model, block_size=4):
        return KVCache.for_model(model.config, num_blocks=4096, block_size=block_size, dtype=model.dtype, device="cpu")

    draft_model = copy.deepcopy(tiny)
    draft_model.model.layers = draft_model.model.layers[:1]
    draft_model.config.num_hidden_layers = 1
    prompts = random_prompts(24, 256, seed=10)
    rep = [[3, 1, 4, 1, 5, 9, 2, 6] * 3]
    res = {"prompts": prompts, "repetitive": rep, "max_new": 24}
    res["plain"] = [cached_autoregressive.generate(tiny, new_cache(tiny), p, 24) for p in prompts + rep]
    for name, make in (("ngram", lambda: NGramDraft(256)),
                       ("draft", lambda: ModelDraft(draft_model, new_cache(draft_model)))):
        for k in (1, 4):
            o, st = generate(tiny, new_cache(tiny), make(), prompts + rep, 24, k=k)
            res[f"{name}_k{k}"] = {"outputs": o, "rounds": st.rounds, "drafted": st.drafted,
                                   "accepted": st.accepted, "attempts": st.attempts, "accepts": st.accepts,
                                   "emitted_per_round": st.emitted_per_round,
                                   "drafted_per_round": st.drafted_per_round}
    # sampled (T = 1) with a seeded generator: the model draft, batch of 6
    o, st = generate(tiny, new_cache(tiny), ModelDraft(draft_model, new_cache(draft_model)), prompts[:6], 16, k=3,
                     temperature=1.0, generator=torch.Generator().manual_seed(5))
    res["sampled_draft_k3"] = {"outputs": o, "accepted": st.accepted, "drafted": st.drafted}
    (OUT / "generate.json").write_text(json.dumps(res))
    print("golden vectors written to", OUT)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/speculative-decoder")
    main(sys.argv[1])
