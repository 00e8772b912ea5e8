"""Host-side pieces of bench.py's measurement contract, on the CPU: the clock samples taken during
the timed region (median SM clock, the throttle reasons that invalidate a run) and the roofline
denominator (the measured peak, or the stated fallback)."""
from __future__ import annotations

import importlib.util
import json

import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def bench_main():
    spec = importlib.util.spec_from_file_location("bench_main", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _clocks_with(bench_main, tmp_path, lines: list[str]):
    c = bench_main.Clocks(0)
    c.path = str(tmp_path / "clocks.csv")
    (tmp_path / "clocks.csv").write_text("\n".join(lines) + "\n")
    return c.summary()


def test_clock_summary_median_and_no_reasons(bench_main, tmp_path) -> None:
    rows = [f"0, {mhz}, 1965, 600.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active"
            for mhz in (1965, 1950, 1965, 1800, 1965)]
    s = _clocks_with(bench_main, tmp_path, rows + ["garbage line", "0, [N/A], 1965, 1, 0x0"])
    assert s == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 5}


def test_clock_summary_reports_throttle_reasons(bench_main, tmp_path) -> None:
    rows = ["0, 1350, 1965, 1001.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
            "0, 1200, 1965, 990.0, 0x0000000000000048, Active, Not Active, Active, Not Active",
            "0, 1965, 1965, 500.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active"]
    s = _clocks_with(bench_main, tmp_path, rows)
    assert s["sm_mhz"] == 1350.0 and s["samples"] == 3
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap", "sw_thermal_slowdown"]


def test_missing_sampler_output_is_reported(bench_main, tmp_path) -> None:
    c = bench_main.Clocks(0)
    c.path = str(tmp_path / "never_written.csv")
    assert c.summary()["reasons"] == ["nvidia-smi unavailable"]


def test_peak_is_the_measured_copy_bandwidth_or_the_stated_fallback(bench_main, tmp_path, monkeypatch) -> None:
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6580.9, "bf16_tflops": 1656.8}))
    monkeypatch.setattr(bench_main, "ROOT", tmp_path)
    assert bench_main.peaks() == {"hbm_gbs": 6580.9, "source": "measured"}
    (tmp_path / "MEASURED_PEAKS.json").unlink()
    assert bench_main.peaks() == {"hbm_gbs": 6650.0, "source": "fallback"}
