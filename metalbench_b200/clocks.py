"""nvidia-smi clock sampling during a timed region.

Started before and stopped after the timed launches; ``summary()`` gives the
median SM clock under load, the maximum clock, the throttle reasons seen
(hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap) and a
verdict: a run that saw one of the first three, or SM clocks stuck well below
the maximum with no reason (a leftover clock lock), is ``rejected``;
sw_power_cap alone is normal for a 1 kW part under load and is only noted.
"""
from __future__ import annotations

import statistics
import subprocess
import threading

REJECT_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return summarize(sm, mx, reasons)


def summarize(sm: list[float], mx, reasons: set) -> dict:
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0,
                "rejected": None}
    med = statistics.median(sm)
    pinned_low = bool(mx) and med < 0.8 * mx and not reasons
    throttled = any(r in reasons for r in REJECT_REASONS)
    return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
            "throttled": throttled, "pinned_low": pinned_low, "rejected": throttled or pinned_low}


class NvmlSampler:
    """The same record from NVML (read only), polled every `period_s` by a
    thread: short per-kernel timed regions of a few tens of milliseconds still
    get samples. Falls back to no samples when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, gpu_index: int, period_s: float = 0.002):
        self.gpu, self.period = gpu_index, period_s
        self.sm: list[float] = []
        self.mx = None
        self.reasons: set = set()
        self._stop = threading.Event()
        self._t = None
        self._nv = None

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self._nv = nv
            self._h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.mx = float(nv.nvmlDeviceGetMaxClockInfo(self._h, nv.NVML_CLOCK_SM))
        except Exception:
            self._nv = None
            return
        self._t = threading.Thread(target=self._poll, daemon=True)
        self._t.start()

    def _poll(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)))
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, attr in self.REASONS:
                    if bits & getattr(nv, attr):
                        self.reasons.add(name)
            except Exception:
                return
            self._stop.wait(self.period)

    def stop(self):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)
        if self._nv is not None:
            try:
                self._nv.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        return summarize(self.sm, self.mx, self.reasons)
