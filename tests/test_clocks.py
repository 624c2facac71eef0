"""The clock sampler against a fake NVML: it summarises and it never calls a setter (CPU)."""
import sys
import time
import types


class _FakeNvml(types.ModuleType):
    NVML_CLOCK_SM = 1

    def __init__(self):
        super().__init__("pynvml")
        self.calls = []
        self._clock = iter([1965.0, 1900.0, 1320.0] + [1965.0] * 10_000)

    def __getattr__(self, name):  # any other NVML entry point, setters and resets included, is refused
        raise AssertionError(f"unexpected NVML call {name}")

    def nvmlInit(self):
        self.calls.append("init")

    def nvmlDeviceGetHandleByUUID(self, uuid):
        raise RuntimeError("no uuid")

    def nvmlDeviceGetHandleByIndex(self, i):
        return ("gpu", i)

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetClockInfo(self, h, kind):
        return next(self._clock)

    def nvmlDeviceGetPowerUsage(self, h):
        return 950_000

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return 0x4


def test_clock_sampler_summarises_read_only(monkeypatch):
    fake = _FakeNvml()
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    from flare_b200.utils.clocks import ClockSampler

    s = ClockSampler(0, interval_s=0.001).start()
    deadline = time.time() + 5.0  # wait for samples, not for a fixed time (a loaded host is slow)
    while len(s.samples) < 3 and time.time() < deadline:
        time.sleep(0.01)
    out = s.stop()
    assert s.error is None, s.error
    assert out["samples"] >= 3 and out["sm_max_mhz"] == 1965.0 and out["reasons"] == ["sw_power_cap"]
    assert out["sm_mhz"] == 1965.0 and out["power_w_max"] == 950.0
