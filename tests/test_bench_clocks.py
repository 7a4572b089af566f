"""bench.py's clock record (CPU, no GPU): the nvidia-smi samples taken inside a timed region are
summarised into the line's `clocks` / `e2e_clocks` (median SM clock, max clock, throttle reasons),
each region separately, with the sampler running across both."""

from __future__ import annotations

import time

import bench


def _line(sm, power_cap="Not Active", thermal="Not Active"):
    # index, clocks.sm, clocks.max.sm, power.draw, reasons.active, hw_slowdown, hw_thermal, sw_thermal, sw_power_cap
    return f"0, {sm}, 1965, 990.0, 0x4, Not Active, Not Active, {thermal}, {power_cap}"


class _Proc:
    def terminate(self):
        self.terminated = True

    def wait(self, timeout=None):
        return 0


def test_regions_are_summarised_separately():
    s = bench.ClockSampler(0)
    s.proc = _Proc()
    t0 = time.monotonic()
    s.lines = [(t0 - 5.0, _line(1965))]  # warm-up, before the first region
    s.begin()
    now = time.monotonic()
    s.lines += [(now + 0.01, _line(1400, power_cap="Active")), (now + 0.02, _line(1420, power_cap="Active")),
                (now + 0.03, _line(1440, power_cap="Active"))]
    first = s.stop()
    assert first["sm_mhz"] == 1420 and first["sm_max_mhz"] == 1965
    assert first["reasons"] == ["sw_power_cap"] and first["samples"] == 3 and first["window"] == "timed region"
    s.begin()
    now = time.monotonic()
    s.lines += [(now + 0.01, _line(1500, thermal="Active"))]
    second = s.stop()
    assert second["sm_mhz"] == 1500 and second["reasons"] == ["sw_thermal_slowdown"] and second["samples"] == 1
    s.close()
    assert s.proc.terminated


def test_a_region_shorter_than_one_sample_says_so():
    s = bench.ClockSampler(0)
    s.proc = _Proc()
    s.lines = [(time.monotonic() - 1.0, _line(1700))]
    s.begin()
    out = s.stop()
    assert out["sm_mhz"] == 1700 and "shorter than one sample" in out["window"]


def test_no_nvidia_smi_is_reported():
    s = bench.ClockSampler(0)
    assert s.stop()["reasons"] == ["nvidia-smi unavailable"]
    s.close()  # nothing to stop
