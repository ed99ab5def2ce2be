"""bench.py's host logic on the CPU: the clock record keeps only the samples taken inside the timed region, reports
their median SM clock, the max clock and every throttle reason seen there, and says "unsampled" when none fell
inside (a run without a clock record cannot be checked for throttling)."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _clocks(samples, t0, t1):
    c = bench.Clocks(0)
    c.samples = samples
    c.t0, c.t1 = t0, t1
    c.source = "test"
    return c.summary()


def test_only_samples_inside_the_timed_region_count():
    s = [(0.9, 1000.0, 1965.0, ["hw_slowdown"]),           # before the region: ignored
         (1.0, 1800.0, 1965.0, []),
         (1.5, 1900.0, 1965.0, ["sw_power_cap"]),
         (2.0, 1965.0, 1965.0, []),
         (2.1, 900.0, 1965.0, ["hw_thermal_slowdown"])]   # after it: ignored
    r = _clocks(s, 1.0, 2.0)
    assert r["samples"] == 3
    assert r["sm_mhz"] == 1900.0 and r["sm_max_mhz"] == 1965.0
    assert r["reasons"] == ["sw_power_cap"]


def test_a_region_without_samples_is_reported_unsampled():
    r = _clocks([(5.0, 1965.0, 1965.0, [])], 1.0, 2.0)
    assert r["samples"] == 0 and r["reasons"] == ["unsampled"] and r["sm_mhz"] is None


def test_reason_bits_name_the_nvml_clock_event_reasons():
    # HwSlowdown 0x8, HwThermalSlowdown 0x40, SwThermalSlowdown 0x20, SwPowerCap 0x4 (nvml.h)
    assert dict(zip(bench.Clocks.NAMES, bench.Clocks.BITS)) == {
        "hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}
