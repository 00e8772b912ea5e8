"""TTFT, TPOT and end-to-end latency of generate() requests, as p50/p95/p99 per configuration.

The definitions are the reference's (bench/latency.py:1-29, `summarize` at 52-87). All times are
seconds from the request's start, taken after a device sync (bench.harness.Stopwatch):

- TTFT: to the "first_token" mark. generate() emits it after the target's prefill and the
  first-token sampler, before the draft does anything.
- TTFT (first round): to the "first_round" mark, the end of the first speculative round
  (target prefill, draft prefill, k draft steps, the first verify and accept); equal to TTFT
  when a workload has no such mark.
- TPOT: (total - TTFT) / (tokens - 1), once for each TTFT definition; requests of one token
  have none.
- draft prefill: from "first_token" to "draft_prefilled".
- end-to-end: the whole request.
`tpot_ms_first_rounds_p50` / `tpot_ms_last_rounds_p50` are medians over the first and the last
`edge_rounds` measured rounds; their ratio shows drift of the machine over the run.
"""
from __future__ import annotations

import math
import statistics
from collections.abc import Iterable, Sequence

from bench.harness import Run, Sample


def percentile(values: Sequence[float], q: float) -> float:
    """The q-th percentile with linear interpolation between the two nearest ranks (numpy's
    default method): position (n - 1) * q / 100 in the sorted values."""
    if len(values) == 0:
        raise ValueError("percentile of no values")
    xs = sorted(values)
    pos = (len(xs) - 1) * q / 100.0
    lo = math.floor(pos)
    hi = min(lo + 1, len(xs) - 1)
    return xs[lo] + (pos - lo) * (xs[hi] - xs[lo])


def spread(values: Sequence[float]) -> dict[str, float]:
    return {"p50": percentile(values, 50), "p95": percentile(values, 95), "p99": percentile(values, 99)}


def _ms(values: Iterable[float | None]) -> dict[str, float] | None:
    kept = [v for v in values if v is not None]
    return spread(kept) if kept else None


def _ttft_first_round(s: Sample) -> float:
    return s.marks.get("first_round", s.ttft)


def _tpot_ms(s: Sample, ttft: float) -> float | None:
    if s.tokens <= 1:
        return None
    return (s.total - ttft) / (s.tokens - 1) * 1e3


def summarize(run: Run, edge_rounds: int = 1) -> dict[str, dict]:
    """Per configuration (in order of first appearance): sample count, token counts and each
    latency in milliseconds as p50/p95/p99."""
    out: dict[str, dict] = {}
    configs = list(dict.fromkeys(s.config for s in run.samples))
    first = set(range(edge_rounds))
    last = set(range(run.repeats - edge_rounds, run.repeats))
    for name in configs:
        ss = [s for s in run.samples if s.config == name]

        def edge_median(rounds: set[int]) -> float | None:
            vals = [_tpot_ms(s, s.ttft) for s in ss if s.round in rounds and s.tokens > 1]
            return statistics.median(vals) if vals else None

        out[name] = {
            "n": len(ss),
            "tokens": _ms(s.tokens for s in ss),
            "ttft_ms": _ms(s.ttft * 1e3 for s in ss),
            "ttft_first_round_ms": _ms(_ttft_first_round(s) * 1e3 for s in ss),
            "tpot_ms": _ms(_tpot_ms(s, s.ttft) for s in ss),
            "tpot_first_round_ms": _ms(_tpot_ms(s, _ttft_first_round(s)) for s in ss),
            "draft_prefill_ms": _ms((s.marks["draft_prefilled"] - s.ttft) * 1e3
                                    for s in ss if "draft_prefilled" in s.marks),
            "e2e_ms": _ms(s.total * 1e3 for s in ss),
            "tpot_ms_first_rounds_p50": edge_median(first),
            "tpot_ms_last_rounds_p50": edge_median(last),
        }
    return out
