"""bench.py's clock record on the CPU, against a fake NVML module.

The benchmark samples SM clocks and throttle reasons in-process through NVML
(read-only queries) and reports, for every measurement, only the samples taken
inside its timed regions: idle pauses, input set-up and warm-up launches before
a timed loop must not enter the median or the reasons. No GPU is touched.
"""

import sys
import threading
import time
import types

import pytest

import bench


class _FakeNvml(types.ModuleType):
    """NVML stand-in whose SM clock and reason bits the test switches."""

    NVML_CLOCK_SM = 1

    def __init__(self):
        super().__init__("pynvml")
        self.lock = threading.Lock()
        self.clock, self.reasons = 1965, 0

    def set(self, clock, reasons):
        with self.lock:
            self.clock, self.reasons = clock, reasons

    def nvmlInit(self):
        pass

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        return object()

    def nvmlDeviceGetHandleByIndex(self, index):
        return object()

    def nvmlDeviceGetMaxClockInfo(self, handle, kind):
        return 1965

    def nvmlDeviceGetClockInfo(self, handle, kind):
        with self.lock:
            return self.clock

    def nvmlDeviceGetCurrentClocksEventReasons(self, handle):
        with self.lock:
            return self.reasons


@pytest.fixture
def fake_nvml(monkeypatch):
    fake = _FakeNvml()
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    return fake


def test_record_keeps_only_timed_window_samples(fake_nvml):
    sampler = bench.ClockSampler(0)
    fake_nvml.set(1200, 0x4)  # an idle pause at low clocks, power cap flagged
    sampler.start()
    assert sampler.source == "nvml 5 ms"
    time.sleep(0.08)
    fake_nvml.set(1965, 0)  # the timed region
    time.sleep(0.01)
    t0 = time.monotonic()
    time.sleep(0.06)
    t1 = time.monotonic()
    time.sleep(0.01)
    fake_nvml.set(1100, 0x40)  # after the region: thermal slowdown must not show
    time.sleep(0.05)
    rec = sampler.stop([(t0, t1)])
    assert rec["timed_windows_only"] is True
    assert rec["sm_mhz"] == 1965
    assert rec["reasons"] == []
    assert rec["samples"] >= 4  # 60 ms at a 5 ms period
    assert rec["sm_max_mhz"] == 1965


def test_record_without_window_samples_reports_all(fake_nvml):
    sampler = bench.ClockSampler(0)
    fake_nvml.set(1700, 0x4)
    sampler.start()
    time.sleep(0.04)
    rec = sampler.stop([(0.0, 1e-9)])  # a window no sample falls into
    assert rec["timed_windows_only"] is False
    assert rec["samples"] >= 1
    assert rec["sm_mhz"] == 1700
    assert rec["reasons"] == ["sw_power_cap"]


def test_time_loop_records_its_window(monkeypatch):
    # time_loop's host-side bookkeeping with CUDA events replaced by stand-ins.
    class _Event:
        def __init__(self, enable_timing=False):
            self.t = None

        def record(self, stream=None):
            self.t = time.monotonic()

        def elapsed_time(self, other):
            return (other.t - self.t) * 1e3

    cuda = types.SimpleNamespace(Event=_Event, synchronize=lambda: None, current_stream=lambda: None)
    monkeypatch.setitem(sys.modules, "torch", types.SimpleNamespace(cuda=cuda))
    n0 = len(bench.TIMED_WINDOWS)
    ms = bench.time_loop(lambda: time.sleep(0.002), steps=5, warmup=1)
    assert len(bench.TIMED_WINDOWS) == n0 + 1
    t0, t1 = bench.TIMED_WINDOWS[-1]
    assert t1 - t0 >= 0.009 and ms >= 1.5
