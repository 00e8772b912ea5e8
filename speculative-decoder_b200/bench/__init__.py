"""Latency reporting for generate(): the timing harness (bench.harness) and the TTFT / TPOT /
end-to-end definitions with their percentile summaries (bench.latency), API-compatible with the
reference's bench package (bench/harness.py, bench/latency.py)."""
