"""Read-only SM clock / throttle-reason sampler (NVML) for the benchmark's timed region.

It only reads: clocks, power and the active clocks-event reasons.  It never sets clocks,
power limits or any other GPU setting.
"""
from __future__ import annotations

import statistics
import threading
import time


class ClockSampler:
    REASONS = {
        "gpu_idle": "nvmlClocksEventReasonGpuIdle",
        "applications_clocks_setting": "nvmlClocksEventReasonApplicationsClocksSetting",
        "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
        "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
        "sync_boost": "nvmlClocksEventReasonSyncBoost",
        "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
        "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
        "hw_power_brake_slowdown": "nvmlClocksEventReasonHwPowerBrakeSlowdown",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.period = period_s
        self.samples: list[tuple[float, int, int]] = []  # (time, sm_mhz, reasons bitmask)
        self._stop = threading.Event()
        self._thread = None
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: report clocks as unavailable
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            self._stop.wait(self.period)

    def start(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self, t0: float | None = None, t1: float | None = None):
        if self._nv is None:
            return None
        s = [x for x in self.samples if (t0 is None or x[0] >= t0) and (t1 is None or x[0] <= t1)]
        if not s:
            s = self.samples[-3:]
        if not s:
            return None
        mask = 0
        for _, _, r in s:
            mask |= r
        reasons = [name for name, attr in self.REASONS.items()
                   if mask & getattr(self._nv, attr, 0) and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(m for _, m, _ in s), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(s)}
