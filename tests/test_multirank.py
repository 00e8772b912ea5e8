"""Request sharding on CPU ranks (gloo, world size 2): contiguous shards, one gather of
tokens and statistics, results identical to one process running every request. The engine's
round itself needs a GPU; here `run` is a deterministic stand-in with the same return type."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spec.loop import SpecStats
from specb200.shard import gather_results, generate_sharded, merge_stats, shard_range

K = 4


def fake_generate(prompts: list[list[int]]) -> tuple[list[list[int]], SpecStats]:
    """Per-request outputs and statistics that depend only on the request itself, with the
    batch semantics of spec.loop.generate: the batch runs as many rounds as its longest
    request needs, and the per-(sequence, round) lists are filled round by round."""
    st = SpecStats(k=K)
    outs, lengths = [], []
    for p in prompts:
        n = 1 + (sum(p) % 7)
        lengths.append(n)
        outs.append([(p[0] * 31 + i) % 1000 for i in range(n)])
        st.drafted += K * n
        st.accepted += sum(p) % (K * n + 1)
        st.attempts = [a + n for a in st.attempts]
        st.accepts = [a + (sum(p) >> i) % 2 for i, a in enumerate(st.accepts)]
    st.rounds = max(lengths, default=0)
    for r in range(st.rounds):
        for b, n in enumerate(lengths):
            if r < n:
                st.emitted_per_round.append(1 + (b + r) % 3)
                st.drafted_per_round.append((b + r) % 3)
    return outs, st


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, prompts: list[list[int]], q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        out, st = generate_sharded(prompts, K, fake_generate)
        q.put((rank, out, st.rounds, st.drafted, st.accepted, st.attempts, st.accepts, st.emitted_per_round))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_prompts", [5, 1])
def test_two_rank_shard_and_gather_match_one_process(n_prompts):
    """5 requests over 2 ranks (3 + 2) and 1 request (one rank idle, still in the gather)."""
    prompts = [[(7 * i + j) % 97 + 1 for j in range(3 + i)] for i in range(n_prompts)]
    want_out, want_st = fake_generate(prompts)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out, rounds, drafted, accepted, attempts, accepts, emitted in results:
        assert out == want_out, rank
        assert (rounds, drafted, accepted) == (want_st.rounds, want_st.drafted, want_st.accepted)
        assert attempts == want_st.attempts and accepts == want_st.accepts
        # the same (sequence, round) entries, grouped by rank rather than interleaved by round
        assert sorted(emitted) == sorted(want_st.emitted_per_round)


def test_shard_range_covers_requests_once():
    for n in range(0, 20):
        for world in range(1, 9):
            got = [i for r in range(world) for i in range(*shard_range(n, r, world))]
            assert got == list(range(n))
            sizes = [shard_range(n, r, world)[1] - shard_range(n, r, world)[0] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_merge_stats_takes_the_longest_round_count():
    _, sa = fake_generate([[1, 2, 3]])
    _, sb = fake_generate([[4, 5]])
    assert sa.rounds != sb.rounds
    m = merge_stats([sa, sb])
    _, want = fake_generate([[1, 2, 3], [4, 5]])
    assert m.rounds == max(sa.rounds, sb.rounds) == want.rounds
    assert (m.drafted, m.accepted, m.attempts, m.accepts) == (want.drafted, want.accepted, want.attempts, want.accepts)
    assert m.emitted_per_round == sa.emitted_per_round + sb.emitted_per_round
    assert sorted(m.emitted_per_round) == sorted(want.emitted_per_round)
    with pytest.raises(ValueError):
        merge_stats([SpecStats(k=2), SpecStats(k=3)])


def test_gather_single_process_group():
    """World size 1 (the driver's N=1 run): the gather is the identity."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        out, st = fake_generate([[3, 1], [9, 9, 9]])
        got_out, got_st = gather_results(out, st)
        assert got_out == out and got_st.accepted == st.accepted and got_st.attempts == st.attempts
    finally:
        dist.destroy_process_group()
