"""Host logic of bench.py that needs no GPU: the roofline denominator each figure is taken against."""
import importlib
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture()
def bench(monkeypatch, tmp_path):
    monkeypatch.syspath_prepend(ROOT)
    mod = importlib.import_module("bench")
    monkeypatch.setattr(mod, "ROOT", str(tmp_path))
    return mod


def _write_peaks(path, **kw):
    with open(os.path.join(path, "MEASURED_PEAKS.json"), "w") as f:
        json.dump(kw, f)


def test_short_timed_region_uses_the_burst_bf16_peak(bench, tmp_path):
    _write_peaks(tmp_path, bf16_tflops=1658.2, bf16_tflops_sustained=1419.7, hbm_gbs=6346.3)
    assert bench._peak_tflops(0.05) == (1658.2, "measured (burst)")
    assert bench._peak_tflops() == (1658.2, "measured (burst)")


def test_long_timed_region_uses_the_sustained_bf16_peak(bench, tmp_path):
    _write_peaks(tmp_path, bf16_tflops=1658.2, bf16_tflops_sustained=1419.7, hbm_gbs=6346.3)
    assert bench._peak_tflops(2.3) == (1419.7, "measured (sustained)")


def test_without_a_sustained_figure_the_burst_one_stands(bench, tmp_path):
    _write_peaks(tmp_path, bf16_tflops=1592.6, hbm_gbs=6437.9)
    assert bench._peak_tflops(2.3) == (1592.6, "measured (burst)")


def test_without_measured_peaks_the_fallbacks_are_named(bench):
    assert bench._peak_tflops(0.1) == (1590.0, "fallback (burst)")
    assert bench._peak_tflops(5.0) == (1400.0, "fallback (sustained)")


def _fake_nvml(monkeypatch, bench, reasons):
    """A stand-in NVML module: 1.9 GHz SM clock, 0.3 ms a read, `reasons` as the event reasons."""
    import time
    import types
    nv = types.ModuleType("pynvml")
    nv.NVML_CLOCK_SM = 1
    nv.nvmlInit = lambda: None
    nv.nvmlDeviceGetHandleByIndex = lambda i: "gpu"
    nv.max_reads = 0

    def max_clock(handle, kind):
        nv.max_reads += 1
        return 1965

    def clock(handle, kind):
        time.sleep(0.0003)
        return 1900

    nv.nvmlDeviceGetMaxClockInfo = max_clock
    nv.nvmlDeviceGetClockInfo = clock
    nv.nvmlDeviceGetCurrentClocksEventReasons = reasons
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    monkeypatch.setattr(bench.torch.cuda, "_get_nvml_device_index", lambda g: 0)
    return nv


def test_clock_sampler_covers_a_region_of_a_few_milliseconds(bench, monkeypatch):
    import time
    nv = _fake_nvml(monkeypatch, bench, lambda h: 0x4 | 0x1)
    with bench.ClockSampler(0) as clk:
        time.sleep(0.008)
    s = clk.summary()
    assert s["samples"] >= 5 and s["sm_mhz"] == 1900 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]  # gpu_idle is not a throttle reason
    assert nv.max_reads == 1  # the maximum clock is fixed: read once


def test_clock_sampler_backs_off_when_reads_fail(bench, monkeypatch):
    import time

    def broken(handle):
        raise RuntimeError("not supported")

    nv = _fake_nvml(monkeypatch, bench, broken)
    nv.reads = 0

    def instant_clock(handle, kind):
        nv.reads += 1
        return 1900

    nv.nvmlDeviceGetClockInfo = instant_clock
    with bench.ClockSampler(0) as clk:
        time.sleep(0.02)
    assert clk.summary()["samples"] == 0
    assert nv.reads <= 40  # about one attempt a millisecond, not a spin
