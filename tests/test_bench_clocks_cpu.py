"""bench.py's clock record against a fake NVML (reading only; nothing touches a GPU): a timed region
shorter than the sampling thread's period still gets samples from the synchronous poll, and the
throttle-reason bits are named."""
import time

import bench


class _FakeNvml:
    NVML_CLOCK_SM = 0

    def nvmlDeviceGetClockInfo(self, h, clock):
        return 1965

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return 0x4  # sw_power_cap


class _FakeEvent:
    """Completes after `n` queries, as a CUDA event does once the queued steps are done."""

    def __init__(self, n):
        self.n = n

    def query(self):
        self.n -= 1
        return self.n < 0


def test_short_timed_region_gets_samples():
    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.samples, s.reasons, s.ok, s.nv, s.h, s.max_mhz = [], set(), True, _FakeNvml(), None, 1965
    s.samples.append((time.perf_counter() - 1.0, 1000, 0))  # a sample from before the region
    t0 = time.perf_counter()
    s.sample_while(_FakeEvent(3), period=0)
    t1 = time.perf_counter()
    summary = s.summary(t0, t1)
    assert summary["samples_in_timed_region"] == 3
    assert summary["sm_mhz"] == 1965 and summary["reasons"] == ["sw_power_cap"]


def test_sampler_without_nvml_is_inert():
    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.samples, s.ok = [], False
    s.sample_while(_FakeEvent(5), period=0)
    assert s.samples == []
