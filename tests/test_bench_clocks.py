"""bench.py's clock record against a fake NVML (no GPU): samples from the
start and the end of even a very short timed region, throttle reasons
collected from every sample with "gpu_idle" left out of the record, and no
record (zero samples) when NVML cannot be initialised."""
import sys
import time
import types

import pytest


def _fake_nvml(mhz=1965, reasons=0x4, fail_init=False):
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    calls = {"clock": 0}

    def init():
        if fail_init:
            raise RuntimeError("NVML unavailable")

    def clock(h, kind):
        calls["clock"] += 1
        return mhz

    m.nvmlInit = init
    m.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    m.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965
    m.nvmlDeviceGetClockInfo = clock
    m.nvmlDeviceGetCurrentClocksEventReasons = lambda h: reasons
    m.calls = calls
    return m


@pytest.fixture
def bench_with(monkeypatch):
    def make(**kw):
        fake = _fake_nvml(**kw)
        monkeypatch.setitem(sys.modules, "pynvml", fake)
        import bench
        return bench, fake
    return make


def test_short_region_has_start_and_end_samples(bench_with):
    bench, _ = bench_with(mhz=1900, reasons=0x1 | 0x4)
    with bench.ClockSampler(0, period=10.0) as clk:  # no periodic sample can land
        pass
    rec = clk.record()
    assert rec["samples"] == 2
    assert rec["sm_mhz"] == 1900 and rec["sm_max_mhz"] == 1965
    assert rec["reasons"] == ["sw_power_cap"]  # gpu_idle is not a throttle reason


def test_periodic_samples_during_region(bench_with):
    bench, fake = bench_with(reasons=0x8)
    with bench.ClockSampler(0, period=0.002) as clk:
        time.sleep(0.05)
    rec = clk.record()
    assert rec["samples"] >= 4
    assert rec["samples"] == fake.calls["clock"]
    assert rec["reasons"] == ["hw_slowdown"]


def test_no_nvml_no_record(bench_with):
    bench, _ = bench_with(fail_init=True)
    with bench.ClockSampler(0) as clk:
        pass
    rec = clk.record()
    assert rec["samples"] == 0 and rec["sm_mhz"] is None
