"""CPU checks of the clock sampler the benchmark attaches to its JSON line, against a fake NVML:
median SM clock over the busy samples, throttle reasons decoded from the event bitmask (idle
excluded), and an "unavailable" summary when NVML cannot start.  The sampler only reads."""
from __future__ import annotations

import sys
import time
import types

import pytest

from femtotron_b200.utils.clocks import ClockSampler


def fake_nvml(samples, *, fail_init=False, old_api=False, max_mhz=1965):
    """A pynvml stand-in whose device returns the given (sm MHz, mW, reasons) in turn (the last
    one repeats).  It records every call, so a test can check that nothing but reads ran."""
    calls = []
    it = iter(samples)
    state = {"cur": samples[0]}

    def nxt():
        try:
            state["cur"] = next(it)
        except StopIteration:
            pass
        return state["cur"]

    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1

    def init():
        calls.append("init")
        if fail_init:
            raise RuntimeError("no NVML")
    m.nvmlInit = init
    m.nvmlDeviceGetHandleByIndex = lambda i: calls.append(("handle", i)) or object()
    m.nvmlDeviceGetMaxClockInfo = lambda h, k: calls.append("max") or max_mhz

    def clock(h, k):
        calls.append("clock")
        return nxt()[0]
    m.nvmlDeviceGetClockInfo = clock
    m.nvmlDeviceGetPowerUsage = lambda h: calls.append("power") or state["cur"][1]
    if old_api:
        def ev(h):
            raise AttributeError("old driver")
        m.nvmlDeviceGetCurrentClocksEventReasons = ev
    else:
        m.nvmlDeviceGetCurrentClocksEventReasons = lambda h: calls.append("reasons") or state["cur"][2]
    m.nvmlDeviceGetCurrentClocksThrottleReasons = \
        lambda h: calls.append("throttle") or state["cur"][2]
    return m, calls


def run_sampler(monkeypatch, nv, n_expected):
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    with ClockSampler(3, period_s=0.001) as clk:
        t0 = time.time()
        while len(clk.samples) < n_expected and time.time() - t0 < 10:
            time.sleep(0.005)
    return clk


def test_median_over_busy_samples_and_reasons(monkeypatch):
    idle, cap, slow = 0x1, 0x4, 0x8
    seq = [(1965, 80_000, idle), (1350, 990_000, cap), (1400, 1000_000, cap), (1380, 995_000, cap),
           (300, 60_000, idle | cap)]
    nv, calls = fake_nvml(seq + [(1390, 990_000, cap | slow)])
    clk = run_sampler(monkeypatch, nv, len(seq) + 1)
    s = clk.summary()
    busy = [x for x in clk.samples if not x[2] & idle]
    assert s["samples"] == len(busy) >= 4
    assert s["sm_mhz"] == pytest.approx(sorted(x[0] for x in busy)[(len(busy) - 1) // 2], abs=25)
    assert s["sm_max_mhz"] == 1965
    assert s["power_w_max"] == pytest.approx(1000.0)
    assert "gpu_idle" not in s["reasons"]
    assert "sw_power_cap" in s["reasons"] and "hw_slowdown" in s["reasons"]
    assert ("handle", 3) in calls
    # read-only: only the query entry points of the fake were called
    assert {c if isinstance(c, str) else c[0] for c in calls} <= \
        {"init", "handle", "max", "clock", "power", "reasons"}


def test_all_idle_samples_still_summarise(monkeypatch):
    nv, _ = fake_nvml([(1965, 70_000, 0x1)])
    clk = run_sampler(monkeypatch, nv, 3)
    s = clk.summary()
    assert s["sm_mhz"] == 1965 and s["reasons"] == []


def test_older_nvml_throttle_reason_call(monkeypatch):
    nv, calls = fake_nvml([(1400, 900_000, 0x40)], old_api=True)
    clk = run_sampler(monkeypatch, nv, 2)
    assert "throttle" in calls
    assert clk.summary()["reasons"] == ["hw_thermal_slowdown"]


def test_unavailable_without_nvml(monkeypatch):
    nv, _ = fake_nvml([(1400, 900_000, 0)], fail_init=True)
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    with ClockSampler(0, period_s=0.001) as clk:
        time.sleep(0.01)
    assert clk.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
