"""Generate tests/golden/latency.json by running the reference's timing harness and latency
summary (bench/harness.py measure, bench/latency.py summarize and percentile).

    python tests/golden/make_latency_golden.py /path/to/speculative-decoder

The reference is imported read-only in this process only. The workloads are seeded synthetic
request timelines played on a fake clock (time moves only when a workload advances it), so
every duration is exact: per call, the time to the first token, optionally the draft prefill
and the rest of the first round, the remaining time and the token count. The fixture holds the
timelines, the configuration orders `measure` drew, every sample and the summaries.
"""
from __future__ import annotations

import json
import random
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent


class FakeClock:
    def __init__(self) -> None:
        self.now = 0.0

    def __call__(self) -> float:
        return self.now

    def sync(self) -> None:
        pass


def timelines(seed: int, names: list[str], calls: int) -> dict[str, list[list]]:
    rng = random.Random(seed)
    out = {}
    for i, name in enumerate(names):
        rows = []
        for _ in range(calls):
            speculative = i % 2 == 0
            first = round(rng.lognormvariate(-3.0, 0.4), 6)
            prefill = round(rng.uniform(0.005, 0.03), 6) if speculative else None
            first_round = round(rng.uniform(0.01, 0.05), 6) if speculative else None
            tail = round(rng.lognormvariate(-1.5, 0.3), 6)
            tokens = rng.choice([1, 2, 17, 64, 129]) if i == 1 else rng.randint(2, 256)
            rows.append([first, prefill, first_round, tail, tokens])
        out[name] = rows
    return out


def play(clock: FakeClock, rows: list[list]):
    it = iter(rows)

    def workload(watch) -> int:
        first, prefill, first_round, tail, tokens = next(it)
        clock.now += first
        watch.mark("first_token")
        if prefill is not None:
            clock.now += prefill
            watch.mark("draft_prefilled")
        if first_round is not None:
            clock.now += first_round
            watch.mark("first_round")
        clock.now += tail
        return tokens

    return workload


def main(ref: str) -> None:
    sys.path.insert(0, ref)
    from bench.harness import measure
    from bench.latency import percentile, summarize

    cases = []
    for seed, names, warmup, repeats, edge in ((3, ["spec_draft", "cached", "spec_ngram"], 2, 9, 2),
                                               (11, ["a", "b", "c", "d", "e"], 1, 6, 1),
                                               (29, ["only"], 0, 25, 5)):
        tl = timelines(seed, names, warmup + repeats)
        clock = FakeClock()
        run = measure({n: play(clock, tl[n]) for n in names}, warmup=warmup, repeats=repeats, sync=clock.sync,
                      seed=seed, clock=clock)
        cases.append({
            "seed": seed, "names": names, "warmup": warmup, "repeats": repeats, "edge_rounds": edge,
            "timelines": tl, "orders": run.orders,
            "samples": [[s.config, s.round, s.slot, s.total, s.tokens, s.marks] for s in run.samples],
            "summary": summarize(run, edge_rounds=edge),
        })
    rng = random.Random(5)
    pct = []
    for n in (1, 2, 3, 10, 101):
        xs = [rng.uniform(-5, 5) for _ in range(n)]
        pct.append({"values": xs, "q": [0, 1, 25, 50, 90, 95, 99, 100],
                    "want": [percentile(xs, q) for q in (0, 1, 25, 50, 90, 95, 99, 100)]})
    (OUT / "latency.json").write_text(json.dumps({"cases": cases, "percentiles": pct}))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_latency_golden.py /path/to/speculative-decoder")
    main(sys.argv[1])
