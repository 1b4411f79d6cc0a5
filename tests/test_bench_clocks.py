"""bench.py's clock sampler against a fake NVML (CPU): samples are taken on a
host thread while the timed region runs, clock-event reason bits map to the
names the JSON line reports, and nothing but read calls reach NVML."""
import importlib
import os
import sys
import time
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _fake_nvml(reason_bits, calls):
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    m.nvmlClocksEventReasonSwPowerCap = 0x4
    m.nvmlClocksEventReasonHwSlowdown = 0x8
    m.nvmlClocksEventReasonSwThermalSlowdown = 0x20
    m.nvmlClocksEventReasonHwThermalSlowdown = 0x40

    def rec(name, value):
        def f(*a):
            calls.append(name)
            return value() if callable(value) else value
        return f

    m.nvmlInit = rec("nvmlInit", None)
    m.nvmlDeviceGetHandleByUUID = rec("nvmlDeviceGetHandleByUUID", "h")
    m.nvmlDeviceGetHandleByIndex = rec("nvmlDeviceGetHandleByIndex", "h")
    m.nvmlDeviceGetClockInfo = rec("nvmlDeviceGetClockInfo", 1700)
    m.nvmlDeviceGetMaxClockInfo = rec("nvmlDeviceGetMaxClockInfo", 1965)
    m.nvmlDeviceGetCurrentClocksEventReasons = rec("nvmlDeviceGetCurrentClocksEventReasons", reason_bits)
    return m


def test_clock_sampler_reads_reasons(monkeypatch):
    calls = []
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(0x4 | 0x40, calls))
    monkeypatch.syspath_prepend(ROOT)
    bench = importlib.import_module("bench")
    with bench.ClockSampler(0, period_s=0.01) as clk:
        time.sleep(0.1)
    s = clk.summary()
    assert s["source"] == "nvml"
    assert s["samples"] >= 3
    assert s["sm_mhz"] == 1700.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
    assert all(c.startswith("nvmlInit") or c.startswith("nvmlDeviceGet") for c in calls)


def test_clock_sampler_without_reasons(monkeypatch):
    calls = []
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(0, calls))
    monkeypatch.syspath_prepend(ROOT)
    bench = importlib.import_module("bench")
    with bench.ClockSampler(0, period_s=0.01) as clk:
        time.sleep(0.05)
    s = clk.summary()
    assert s["reasons"] == [] and s["samples"] >= 1
