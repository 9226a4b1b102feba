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
