"""bench.py's clock record, checked on CPU against a fake NVML.

The bench samples SM clocks and clock-event reasons while the timed region
runs (a record that saw thermal or hardware slowdown rejects the number).
These tests replace ``pynvml`` with a fake that only answers the read-only
queries the sampler makes, so no GPU and no driver are needed.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import time
import types

import pytest

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUS = "00000000:1B:00.0"


def _load_bench():
    spec = importlib.util.spec_from_file_location("_bench_under_test", os.path.join(_ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _fake_nvml(clocks, reasons, fail_init=False):
    """A module with the NVML calls the sampler uses; clocks and reason
    bitmasks are handed out in turn (the last one repeats)."""
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    m.nvmlClocksEventReasonSwPowerCap = 0x4
    m.nvmlClocksEventReasonHwSlowdown = 0x8
    m.nvmlClocksEventReasonSwThermalSlowdown = 0x20
    m.nvmlClocksEventReasonHwThermalSlowdown = 0x40
    state = {"i": 0, "j": 0, "shutdown": 0}

    def init():
        if fail_init:
            raise RuntimeError("NVML unavailable")

    def clock(handle, kind):
        v = clocks[min(state["i"], len(clocks) - 1)]
        state["i"] += 1
        return v

    def event_reasons(handle):
        v = reasons[min(state["j"], len(reasons) - 1)]
        state["j"] += 1
        return v

    m.nvmlInit = init
    m.nvmlShutdown = lambda: state.__setitem__("shutdown", state["shutdown"] + 1)
    m.nvmlDeviceGetHandleByIndex = lambda i: pytest.fail("the sampler must not open a GPU by NVML index")
    m.nvmlDeviceGetHandleByPciBusId_v2 = lambda bus: state.__setitem__("bus", bus) or ("gpu", bus)
    m.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965
    m.nvmlDeviceGetClockInfo = clock
    m.nvmlDeviceGetCurrentClocksEventReasons = event_reasons
    m.state = state
    return m


def test_nvml_samples_clocks_and_reasons(monkeypatch):
    bench = _load_bench()
    fake = _fake_nvml([1965, 1965, 1800, 1965], [0, 0x4, 0x4, 0])
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(BUS, period_s=0.005) as c:
        assert c.samples, "__enter__ returns only after the first sample"
        deadline = time.perf_counter() + 5.0
        while len(c.samples) < 4 and time.perf_counter() < deadline:
            time.sleep(0.01)
    s = c.summary()
    assert fake.state["bus"] == BUS and s["bus_id"] == BUS
    assert s["samples"] >= 4
    assert s["sm_max_mhz"] == 1965.0
    assert s["sm_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
    assert s["sampler"].startswith("nvml")
    assert fake.state["shutdown"] == 1


def test_slowdown_reasons_are_reported(monkeypatch):
    bench = _load_bench()
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml([1200], [0x40 | 0x8 | 0x20]))
    with bench.ClockSampler(BUS, period_s=0.005) as c:
        time.sleep(0.02)
    assert c.summary()["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]


def test_unsampled_without_nvml_or_nvidia_smi(monkeypatch):
    bench = _load_bench()
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml([1965], [0], fail_init=True))

    def no_smi(*a, **k):
        raise OSError("nvidia-smi not found")

    monkeypatch.setattr(bench.subprocess, "Popen", no_smi)
    with bench.ClockSampler(BUS) as c:
        pass
    assert c.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "bus_id": BUS}


def test_nvidia_smi_fallback_names_the_bus_id(monkeypatch):
    bench = _load_bench()
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml([1965], [0], fail_init=True))
    seen = {}

    def fake_popen(cmd, **k):
        seen["cmd"] = cmd
        raise OSError("stop here")

    monkeypatch.setattr(bench.subprocess, "Popen", fake_popen)
    with bench.ClockSampler(BUS):
        pass
    assert seen["cmd"][:3] == ["nvidia-smi", "-i", BUS]


if __name__ == "__main__":
    sys.exit(pytest.main([__file__, "-q"]))
