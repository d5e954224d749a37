"""Sample SM clocks, power and clock-event (throttle) reasons through NVML in a background
thread while a timed region runs.  Read-only: no GPU setting is changed."""
from __future__ import annotations

import statistics
import threading
import time

_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    def __init__(self, device_index: int = 0, period_s: float = 0.2):
        self.device_index = device_index
        self.period_s = period_s
        self.samples: list[tuple[int, float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        self._ok = False

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nv = pynvml
            self._ok = True
        except Exception:
            self._ok = False
            return self
        self._thr = threading.Thread(target=self._run, daemon=True)
        self._thr.start()
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except Exception:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.samples.append((sm, pw, rs))
            except Exception:
                pass
            time.sleep(self.period_s)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr is not None:
            self._thr.join(timeout=2)
        return False

    def summary(self) -> dict:
        if not self._ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        busy = [s for s in self.samples if not (s[2] & 0x1)] or self.samples
        reasons = set()
        for _, _, r in busy:
            for bit, name in _REASONS.items():
                if r & bit and bit != 0x1:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in busy), "sm_max_mhz": self.max_mhz,
                "power_w_max": max(s[1] for s in busy), "reasons": sorted(reasons),
                "samples": len(busy)}
