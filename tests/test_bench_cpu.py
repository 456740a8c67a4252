"""CPU: bench.py's host-side pieces - the clock summary that decides whether a
run is kept, and the modes that have no reference arm."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _line(sm, smax=1965, active="0x0", hw="Not Active", hwt="Not Active", swt="Not Active",
          cap="Not Active"):
    return f"0, {sm}, {smax}, 700.5, {active}, {hw}, {hwt}, {swt}, {cap}"


def test_clock_summary_median_over_loaded_samples():
    lines = [_line(345), _line(1950), _line(1965), _line(1900, cap="Active"), "garbage"]
    c = bench.summarize_clocks(lines)
    assert c["sm_mhz"] == 1950 and c["sm_max_mhz"] == 1965 and c["samples"] == 4
    assert c["reasons"] == ["sw_power_cap"]


@pytest.mark.parametrize("field", ["hw", "hwt", "swt"])
def test_clock_summary_reports_rejecting_reasons(field):
    c = bench.summarize_clocks([_line(1800, **{field: "Active"})])
    assert c["reasons"] == [{"hw": "hw_slowdown", "hwt": "hw_thermal_slowdown",
                             "swt": "sw_thermal_slowdown"}[field]]


def test_clock_summary_without_samples():
    assert bench.summarize_clocks([])["reasons"] == ["no samples"]
    assert bench.summarize_clocks(["0, [N/A], [N/A], 1, 2, 3, 4, 5, 6"])["sm_mhz"] is None


def test_linear_mode_has_no_reference_arm():
    run = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--linear", "--impl",
                          "reference"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert run.returncode == 0, run.stderr[-2000:]
    line = json.loads(run.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line
