"""Read-only GPU clock / throttle-reason sampler (NVML, background thread).

Samples SM clock, max SM clock, power and the active clock-event reasons of
one GPU every ``interval_s`` while a timed region runs.  It only reads NVML;
it never changes a clock, power limit or any other device setting.
"""
from __future__ import annotations

import statistics
import threading
import time

REASON_BITS = {
    "sw_power_cap": 0x4,
    "hw_slowdown": 0x8,
    "sw_thermal_slowdown": 0x20,
    "hw_thermal_slowdown": 0x40,
    "hw_power_brake_slowdown": 0x80,
}


class ClockSampler:
    def __init__(self, torch_device_index: int = 0, interval_s: float = 0.01):
        self.interval_s = interval_s
        self.samples: list[tuple[float, float, float, int]] = []
        self._stop = threading.Event()
        self._thread = None
        self._handle = None
        self._nvml = None
        self.error = None
        try:
            import pynvml as nv
            import torch

            nv.nvmlInit()
            self._nvml = nv
            handle = None
            try:
                uuid = str(torch.cuda.get_device_properties(torch_device_index).uuid)
                handle = nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:  # noqa: BLE001 - fall back to the visible index
                handle = nv.nvmlDeviceGetHandleByIndex(torch_device_index)
            self._handle = handle
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM))
        except Exception as exc:  # noqa: BLE001
            self.error = repr(exc)
            self.max_mhz = None

    def _reasons(self):
        nv = self._nvml
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(fn(self._handle))

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
                pw = float(nv.nvmlDeviceGetPowerUsage(self._handle)) / 1000.0
                self.samples.append((time.perf_counter(), sm, pw, self._reasons()))
            except Exception as exc:  # noqa: BLE001
                self.error = repr(exc)
                return
            time.sleep(self.interval_s)

    def start(self) -> "ClockSampler":
        if self._handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def stop(self) -> dict:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "error": self.error}
        mask = 0
        for s in self.samples:
            mask |= s[3]
        reasons = sorted(n for n, b in REASON_BITS.items() if mask & b)
        return {"sm_mhz": statistics.median(s[1] for s in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples),
                "power_w_max": max(s[2] for s in self.samples)}


__all__ = ["ClockSampler", "REASON_BITS"]
