"""Host-side pieces of bench.py that need no GPU: the clock-sample parser and the CPU baselines."""
from __future__ import annotations

import bench


def test_clock_summary_parses_samples_and_reasons():
    clk = bench.ClockSampler(0)
    clk.lines = [
        "0, 1965, 1965, 700.1, Not Active, Not Active, Not Active, Not Active\n",
        "0, 1950, 1965, 990.5, Not Active, Not Active, Not Active, Active\n",
        "0, 1800, 1965, 995.0, Not Active, Not Active, Not Active, Active\n",
        "garbage line\n",
    ]
    s = clk.summary()
    assert s["samples"] == 3
    assert s["sm_mhz"] == 1950.0
    assert s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_summary_without_samples_reports_error():
    clk = bench.ClockSampler(0)
    clk.error = "No devices were found"
    s = clk.summary()
    assert s["samples"] == 0 and s["sm_mhz"] is None and s["error"] == "No devices were found"


def test_host_threads_ignores_omp_setting(monkeypatch):
    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    assert bench.host_threads() >= 1


def test_cpu_sample_reports_a_timed_bounded_sample():
    r = bench.cpu_sample(bench.host_threads(), seconds=0.05, chunk_blocks=2)
    assert r["kind"] == "port" and r["unit"] == "Gcoords/s"
    assert r["coords"] % (2 * bench.BLOCK) == 0 and r["coords"] > 0
    assert r["value"] > 0 and r["elapsed_s"] >= 0.05
