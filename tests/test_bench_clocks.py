"""bench.py's clock record (the `clocks` object of its JSON line): the
summary of NVML samples and of nvidia-smi lines, with no GPU."""

from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("d3_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_nvml_samples_summary(bench):
    c = bench.ClockSampler(0)
    c.samples = [(1965.0, 1965.0, frozenset()), (1950.0, 1965.0, frozenset({"sw_power_cap"})),
                 (1965.0, 1965.0, frozenset())]
    s = c.summary()
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    assert s["source"].startswith("nvml")


def test_nvidia_smi_lines_summary(bench):
    c = bench.ClockSampler(0)
    c.lines = ["0, 1800, 1965, 700.1, 0x4, Not Active, Active, Not Active, Active",
               "0, 1900, 1965, 710.2, 0x4, Not Active, Not Active, Not Active, Active",
               "garbage"]
    s = c.summary()
    assert s["sm_mhz"] == 1850.0 and s["samples"] == 2
    assert s["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
    assert s["source"].startswith("nvidia-smi")


def test_no_samples(bench):
    s = bench.ClockSampler(0).summary()
    assert s["sm_mhz"] is None and s["samples"] == 0 and s["reasons"] == []
