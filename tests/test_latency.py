"""The latency harness (bench.harness, bench.latency): the reference's own measure/summarize runs
replayed (tests/golden/latency.json), the properties its timing rules promise, and one GPU run
of the engine's generate() through the harness with CUDA synchronisation."""
from __future__ import annotations

import json
import math
import subprocess

import numpy as np
import pytest
import torch

from conftest import GOLDEN

from bench.harness import Stopwatch, environment, measure, synchronizer
from bench.latency import percentile, spread, summarize


class Clock:
    """Fake time: advances only when a workload says so; logs clock reads and syncs."""

    def __init__(self) -> None:
        self.now = 0.0
        self.log: list[str] = []

    def __call__(self) -> float:
        self.log.append("read")
        return self.now

    def sync(self) -> None:
        self.log.append("sync")


def player(clock: Clock, rows: list[list]):
    """Plays the fixture's request timelines (first, draft prefill, first round, tail, tokens)."""
    it = iter(rows)

    def workload(watch: Stopwatch) -> int:
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


def assert_close(got, want, path="") -> None:
    if isinstance(want, dict):
        assert isinstance(got, dict) and set(got) == set(want), path
        for k in want:
            assert_close(got[k], want[k], f"{path}.{k}")
    elif want is None:
        assert got is None, path
    else:
        assert math.isclose(got, want, rel_tol=1e-12, abs_tol=1e-12), (path, got, want)


@pytest.fixture(scope="module")
def golden_latency() -> dict:
    return json.loads((GOLDEN / "latency.json").read_text())


def test_measure_and_summarize_reproduce_reference_runs(golden_latency) -> None:
    """Same seed, same timelines: the same configuration orders, samples and summaries as the
    reference's harness produced."""
    for case in golden_latency["cases"]:
        clock = Clock()
        run = measure({n: player(clock, case["timelines"][n]) for n in case["names"]}, warmup=case["warmup"],
                      repeats=case["repeats"], sync=clock.sync, seed=case["seed"], clock=clock)
        assert run.orders == case["orders"]
        assert len(run.samples) == len(case["samples"])
        for s, (config, rnd, slot, total, tokens, marks) in zip(run.samples, case["samples"]):
            assert (s.config, s.round, s.slot, s.tokens) == (config, rnd, slot, tokens)
            assert_close(s.total, total)
            assert_close(s.marks, marks)
        assert_close(summarize(run, edge_rounds=case["edge_rounds"]), case["summary"])


def test_percentile_matches_reference_and_numpy(golden_latency) -> None:
    for c in golden_latency["percentiles"]:
        for q, want in zip(c["q"], c["want"]):
            assert percentile(c["values"], q) == pytest.approx(want, rel=1e-12, abs=1e-12)
            assert percentile(c["values"], q) == pytest.approx(float(np.percentile(c["values"], q)), abs=1e-9)
    assert spread([4.0]) == {"p50": 4.0, "p95": 4.0, "p99": 4.0}
    with pytest.raises(ValueError):
        percentile([], 50)


def test_known_timeline_gives_exact_ttft_tpot_and_e2e() -> None:
    # prefill 80 ms -> first token; draft prefill 20 ms; first round 40 ms with 4 more tokens;
    # then 11 tokens at 5 ms: 16 tokens, 195 ms in total
    clock = Clock()

    def spec(watch: Stopwatch) -> int:
        clock.now += 0.080
        watch.first_token()
        clock.now += 0.020
        watch.mark("draft_prefilled")
        clock.now += 0.040
        watch.mark("first_round")
        clock.now += 11 * 0.005
        return 16

    s = summarize(measure({"spec": spec}, warmup=1, repeats=3, sync=clock.sync, seed=1, clock=clock))["spec"]
    assert s["n"] == 3
    assert s["ttft_ms"]["p50"] == pytest.approx(80.0)
    assert s["ttft_first_round_ms"]["p50"] == pytest.approx(140.0)
    assert s["draft_prefill_ms"]["p99"] == pytest.approx(20.0)
    assert s["e2e_ms"]["p95"] == pytest.approx(195.0)
    assert s["tpot_ms"]["p50"] == pytest.approx(115.0 / 15)
    assert s["tpot_first_round_ms"]["p50"] == pytest.approx(55.0 / 15)


def test_every_clock_read_follows_a_sync_and_marks_keep_the_first() -> None:
    clock = Clock()

    def twice(watch: Stopwatch) -> int:
        clock.now += 0.01
        watch.first_token()
        clock.now += 0.01
        watch.first_token()  # ignored: no sync, no read
        return 3

    run = measure({"x": twice, "y": twice}, warmup=2, repeats=2, sync=clock.sync, seed=0, clock=clock)
    reads = [i for i, e in enumerate(clock.log) if e == "read"]
    assert len(reads) == 3 * 2 * (2 + 2)  # start, first token, stop; 2 configs; warm-up + measured
    assert all(clock.log[i - 1] == "sync" for i in reads)
    assert all(s.ttft == pytest.approx(0.01) for s in run.samples)


def test_warmup_is_per_configuration_and_unmeasured() -> None:
    clock = Clock()
    calls = {"p": 0, "q": 0}

    def make(name: str):
        def w(watch: Stopwatch) -> int:
            calls[name] += 1
            clock.now += 3.0 if calls[name] <= 3 else 0.002
            watch.first_token()
            return 1
        return w

    run = measure({n: make(n) for n in calls}, warmup=3, repeats=4, sync=clock.sync, seed=2, clock=clock)
    assert calls == {"p": 7, "q": 7}
    assert all(s.total == pytest.approx(0.002) for s in run.samples)
    assert sorted((s.round, s.slot) for s in run.samples) == [(r, i) for r in range(4) for i in range(2)]


def test_orders_are_seeded_shuffles() -> None:
    names = ["a", "b", "c", "d", "e"]

    def orders(seed: int) -> list[list[str]]:
        clock = Clock()
        w = player(clock, [[0.001, None, None, 0.001, 2]] * 20)
        return measure({n: w for n in names}, warmup=0, repeats=4, sync=clock.sync, seed=seed, clock=clock).orders

    a = orders(4)
    assert a == orders(4) and all(sorted(o) == names for o in a) and len({tuple(o) for o in a}) > 1
    assert a != orders(5)


def test_workload_without_first_token_is_an_error() -> None:
    with pytest.raises(RuntimeError, match="never reported its first token"):
        measure({"silent": lambda watch: 5}, warmup=0, repeats=1, sync=lambda: None, seed=0)


def test_after_each_runs_outside_the_window() -> None:
    clock = Clock()
    seen: list[tuple[str, int]] = []

    def hook(name: str, rnd: int) -> None:
        clock.now += 100.0
        seen.append((name, rnd))

    run = measure({"a": player(clock, [[0.01, None, None, 0.02, 4]] * 3)}, warmup=1, repeats=2, sync=clock.sync,
                  seed=0, clock=clock, after_each=hook)
    assert seen == [("a", -1), ("a", 0), ("a", 1)]
    assert all(s.total == pytest.approx(0.03) for s in run.samples)


def test_one_token_requests_have_no_tpot() -> None:
    clock = Clock()
    s = summarize(measure({"one": player(clock, [[0.01, None, None, 0.0, 1]] * 2)}, warmup=0, repeats=2,
                          sync=clock.sync, seed=0, clock=clock))["one"]
    assert s["tpot_ms"] is None and s["tpot_ms_first_rounds_p50"] is None
    assert s["ttft_first_round_ms"] == s["ttft_ms"] and s["draft_prefill_ms"] is None


def test_synchronizer_and_environment() -> None:
    assert synchronizer(torch.device("cpu"))() is None
    assert synchronizer(torch.device("cuda")) is torch.cuda.synchronize
    rec = environment(torch.device("cpu"), seed=3, models={"target": "tiny"})
    head = subprocess.run(["git", "rev-parse", "HEAD"], capture_output=True, text=True).stdout.strip() or None
    assert rec["git_commit"] == head
    assert rec["seed"] == 3 and rec["models"] == {"target": "tiny"} and rec["gpu"] is None
    assert {"torch", "transformers", "numpy"} <= set(rec["packages"])


@pytest.mark.gpu
def test_engine_generate_through_the_harness() -> None:
    """generate() on the fused CUDA-graph path, timed by the harness with CUDA syncs: the
    events arrive in the loop's order and the latencies are consistent."""
    from cache.kv import KVCache
    from conftest import early_exit, tiny_fp32
    from spec.draft import ModelDraft
    from spec.loop import generate

    dev = torch.device("cuda")
    tiny = tiny_fp32().to(dev)
    draft = early_exit(tiny)

    def cache(m):
        return KVCache.for_model(m.config, num_blocks=512, block_size=4, dtype=m.dtype, device=dev)

    events: list[list[str]] = []

    def spec(watch: Stopwatch) -> int:
        seen: list[str] = []
        events.append(seen)

        def on_event(e: str) -> None:
            seen.append(e)
            watch.mark(e)

        out, _ = generate(tiny, cache(tiny), ModelDraft(draft, cache(draft)), [[5, 9, 2, 7]], 24, k=4,
                          on_event=on_event)
        return len(out[0])

    env = environment(dev, seed=0)
    assert "sm_100" in env["gpu"] or "SMs" in env["gpu"]
    run = measure({"spec_draft": spec}, warmup=1, repeats=3, sync=synchronizer(dev), seed=0)
    assert all(e == ["first_token", "draft_prefilled", "first_round"] for e in events)
    for s in run.samples:
        assert s.tokens == 24
        assert 0 < s.marks["first_token"] < s.marks["draft_prefilled"] < s.marks["first_round"] <= s.total
    summ = summarize(run)["spec_draft"]
    assert summ["n"] == 3 and summ["tokens"]["p50"] == 24
    assert summ["tpot_ms"]["p50"] > 0 and summ["e2e_ms"]["p50"] >= summ["ttft_first_round_ms"]["p50"]
