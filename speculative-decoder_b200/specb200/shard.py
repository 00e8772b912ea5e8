"""Request sharding across the GPUs of one box: one process per GPU, contiguous request
ranges, no collective inside a round, and one gather of tokens and statistics at the end.

The reference runs every request in one process (spec/loop.py:38-104); requests are fully
independent there (each has its own context, cache sequence and draft state), so splitting
the prompt list into contiguous ranges and concatenating the per-range outputs in rank order
returns exactly what one process would. The statistics counters merge by addition, except
`rounds`: one process steps its whole batch round by round until the longest request is done,
so its round count is the largest of the ranks' counts. The per-(sequence, round) lists
(`emitted_per_round`, `drafted_per_round`) hold the same entries as one process's, grouped by
rank instead of interleaved round by round.

The gather is the only collective: `torch.distributed` all_gather of a padded int64 payload
(NCCL over NVLink on GPUs, gloo on CPU). It runs after the timed region, carries kilobytes,
and every rank takes the same collective steps in the same order.
"""
from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
import torch.distributed as dist

from spec.loop import SpecStats


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous slice [lo, hi) of n requests owned by `rank`: the first n % world ranks
    take one extra request."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _pack(outputs: Sequence[Sequence[int]], stats: SpecStats) -> list[int]:
    """Flatten one rank's results: header, output lengths and tokens, stats counters and the
    per-round lists (all int64)."""
    flat = [len(outputs), stats.k, stats.rounds, stats.drafted, stats.accepted, len(stats.emitted_per_round)]
    flat += [len(o) for o in outputs]
    for o in outputs:
        flat += list(o)
    flat += stats.attempts + stats.accepts + stats.emitted_per_round + stats.drafted_per_round
    return flat


def _unpack(flat: list[int]) -> tuple[list[list[int]], SpecStats]:
    n, k, rounds, drafted, accepted, n_rounds = flat[:6]
    pos = 6
    lens = flat[pos:pos + n]
    pos += n
    outputs = []
    for ln in lens:
        outputs.append(flat[pos:pos + ln])
        pos += ln
    st = SpecStats(k=k)
    st.rounds, st.drafted, st.accepted = rounds, drafted, accepted
    st.attempts = flat[pos:pos + k]
    pos += k
    st.accepts = flat[pos:pos + k]
    pos += k
    st.emitted_per_round = flat[pos:pos + n_rounds]
    pos += n_rounds
    st.drafted_per_round = flat[pos:pos + n_rounds]
    return outputs, st


def merge_stats(parts: Sequence[SpecStats]) -> SpecStats:
    """Sum the counters, take the largest round count (the batch loop of one process runs as
    many rounds as its longest request needs), and concatenate the per-(sequence, round) lists
    in rank order."""
    if not parts:
        raise ValueError("no statistics to merge")
    k = parts[0].k
    out = SpecStats(k=k)
    for st in parts:
        if st.k != k:
            raise ValueError(f"draft length differs across ranks: {st.k} != {k}")
        out.rounds = max(out.rounds, st.rounds)
        out.drafted += st.drafted
        out.accepted += st.accepted
        out.attempts = [a + b for a, b in zip(out.attempts, st.attempts)]
        out.accepts = [a + b for a, b in zip(out.accepts, st.accepts)]
        out.emitted_per_round += st.emitted_per_round
        out.drafted_per_round += st.drafted_per_round
    return out


def gather_results(outputs: Sequence[Sequence[int]], stats: SpecStats, device: torch.device | str = "cpu",
                   group=None) -> tuple[list[list[int]], SpecStats]:
    """All-gather every rank's outputs and statistics; returns (outputs of all ranks in rank
    order, merged statistics) on every rank. Two collectives: the payload lengths, then the
    payloads padded to the longest."""
    world = dist.get_world_size(group)
    mine = torch.tensor(_pack(outputs, stats), dtype=torch.int64, device=device)
    n = torch.tensor([mine.numel()], dtype=torch.int64, device=device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    width = int(max(int(s.item()) for s in sizes))
    padded = torch.zeros(width, dtype=torch.int64, device=device)
    padded[: mine.numel()] = mine
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    all_out: list[list[int]] = []
    all_stats: list[SpecStats] = []
    for p, s in zip(parts, sizes):
        o, st = _unpack(p[: int(s.item())].cpu().tolist())
        all_out += o
        all_stats.append(st)
    return all_out, merge_stats(all_stats)


def generate_sharded(prompts: Sequence[Sequence[int]], k: int,
                     run: Callable[[list[list[int]]], tuple[list[list[int]], SpecStats]],
                     device: torch.device | str = "cpu", group=None) -> tuple[list[list[int]], SpecStats]:
    """Run `run(prompts[lo:hi])` (e.g. a closure over spec.loop.generate with this rank's
    models and cache) on this rank's contiguous share of the requests, then gather. Every
    rank returns the outputs of all requests, in the order of `prompts`; a rank with no
    requests contributes empty results (draft length k) and still joins the gather."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    lo, hi = shard_range(len(prompts), rank, world)
    if hi > lo:
        out, st = run([list(p) for p in prompts[lo:hi]])
    else:
        out, st = [], SpecStats(k=k)
    return gather_results(out, st, device=device, group=group)
