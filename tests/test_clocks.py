"""ClockSampler against a fake NVML (CPU): samples are taken on entry, while running and on exit,
and throttle-reason bits map to the reported names. It only reads; nothing is set."""
import sys
import time
import types


def _fake_nvml(bits):
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    m.calls = []
    m.nvmlInit = lambda: None
    m.nvmlShutdown = lambda: None
    m.nvmlDeviceGetCount = lambda: 2
    m.nvmlDeviceGetHandleByIndex = lambda i: i
    m.nvmlDeviceGetClockInfo = lambda h, k: 1800 + h
    m.nvmlDeviceGetMaxClockInfo = lambda h, k: 1965
    m.nvmlDeviceGetPowerUsage = lambda h: 700000
    m.nvmlDeviceGetUtilizationRates = lambda h: types.SimpleNamespace(gpu=100)
    m.nvmlDeviceGetCurrentClocksEventReasons = lambda h: bits
    return m


def test_clock_sampler_with_fake_nvml(monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(0x4))
    from originccl_b200.utils.clocks import ClockSampler
    with ClockSampler([0], interval_ms=1.0) as cs:
        time.sleep(0.02)
    s = cs.summary()
    assert s["source"] == "nvml" and s["samples"] >= 3
    assert s["sm_mhz"] == 1800 and s["sm_max_mhz"] == 1965 and s["reasons"] == ["sw_power_cap"]


def test_clock_sampler_reports_thermal_reasons(monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(0x40 | 0x8))
    from originccl_b200.utils.clocks import ClockSampler
    with ClockSampler([1], interval_ms=1.0) as cs:
        pass
    assert cs.summary()["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"]


def test_clock_sampler_for_no_gpus_takes_no_samples():
    from originccl_b200.utils.clocks import ClockSampler
    with ClockSampler([]) as cs:
        pass
    assert cs.summary()["samples"] == 0
