"""Host-side parts of the benchmark that need no GPU: the clock sampler over a
fake NVML (read-only queries; nothing is set), including a timed region too
short for the polling interval."""

import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class FakeNVML:
    NVML_CLOCK_SM = 0

    def __init__(self, sm=1965, reasons=0):
        self.sm, self.reasons, self.calls = sm, reasons, 0

    def nvmlDeviceGetMaxClockInfo(self, h, clock):
        return 1965

    def nvmlDeviceGetClockInfo(self, h, clock):
        self.calls += 1
        return self.sm

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return self.reasons


def _sampler(bench, fake):
    c = bench.Clocks(0, None)
    c._nvml = (fake, None)
    return c


def test_zero_length_region_still_sampled(bench):
    fake = FakeNVML(sm=1900)
    c = _sampler(bench, fake)
    with c:
        pass
    s = c.summary()
    assert s["samples"] >= 2 and s["source"] == "nvml"
    assert s["sm_mhz"] == 1900 and s["sm_max_mhz"] == 1965 and s["reasons"] == []


@pytest.mark.parametrize("bits,expect", [
    (0x4, ["sw_power_cap"]),
    (0x8 | 0x40, ["hw_slowdown", "hw_thermal_slowdown"]),
    (0x20, ["sw_thermal_slowdown"]),
    (0x1, []),  # GPU idle: not a slowdown reason
])
def test_reason_bits(bench, bits, expect):
    c = _sampler(bench, FakeNVML(reasons=bits))
    with c:
        pass
    assert c.summary()["reasons"] == expect


def test_failing_queries_report_unsampled(bench):
    class Broken(FakeNVML):
        def nvmlDeviceGetClockInfo(self, h, clock):
            raise RuntimeError("NVML error")

    c = _sampler(bench, Broken())
    with c:
        pass
    assert c.summary()["reasons"] == ["unsampled"]
