"""Host-side helpers of bench.py, on CPU: the FLOP count of the metric, the
peak and traffic files it reads, and the clock record built from nvidia-smi
samples (fed here as text, no GPU or nvidia-smi needed)."""
from __future__ import annotations

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _line(sm, power, cap=False, thermal=False):
    act = lambda b: "Active" if b else "Not Active"  # noqa: E731
    return f"0, {sm}, 1965, {power}, 0x0, Not Active, Not Active, {act(thermal)}, {act(cap)}"


def _stop(lines):
    class _Proc:
        def terminate(self):
            pass

        def wait(self, timeout=None):
            pass

    s = bench.ClockSampler("0")
    s.proc, s.thread, s.lines = _Proc(), None, list(lines)
    return s.stop()


def test_flops_follow_the_metric_convention():
    # 4 * B * Hq * S * S * D, halved under the causal mask.
    assert bench.flops(4, 8192, 32, 128, True) == 4 * 4 * 32 * 8192 * 8192 * 128 / 2
    assert bench.flops(1, 512, 8, 64, False) == 4 * 512 * 512 * 8 * 64


def test_clock_record_uses_loaded_samples_and_reports_reasons():
    rec = _stop([_line(1965, 120.0), _line(1800, 950.0, cap=True), _line(1700, 990.0, cap=True),
                 _line(1965, 130.0)])
    assert rec["samples"] == 4 and rec["samples_under_load"] == 2
    assert rec["sm_mhz"] == 1750.0  # median of the two samples at >= 60 % of the peak power
    assert rec["sm_max_mhz"] == 1965.0 and rec["power_w_max"] == 990.0
    assert rec["reasons"] == ["sw_power_cap"]


def test_clock_record_flags_thermal_slowdown_and_skips_bad_lines():
    rec = _stop(["garbage", _line(1500, 800.0, thermal=True), "0, N/A, 1965, 10, 0x0, a, b, c, d"])
    assert rec["samples"] == 1 and rec["reasons"] == ["sw_thermal_slowdown"]
    assert _stop([]) is None


def test_peaks_and_traffic_files_load():
    peaks, kind = bench.load_peaks()
    assert kind in ("measured", "fallback")
    assert peaks["hbm_gbs"] > 1000 and peaks["bf16_tflops"] > 500
    assert bench.load_traffic("cfg4") > 4e8  # four batches of ~131 MB
