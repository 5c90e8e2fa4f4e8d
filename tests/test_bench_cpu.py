"""CPU checks of bench.py's host-side pieces: the algorithmic bytes of the
headline call, the committed ncu traffic it reports, the peak it divides by,
and the per-CTA timeline summary (synthetic stamps, no GPU)."""

import json
import os

import numpy as np

import bench


def test_algorithmic_bytes_of_the_headline_call():
    # qweight + scales + packed qzeros + LoRA A + LoRA B + x + y
    assert bench.BYTES_PER_CALL == 12_451_840 + 389_120 + 97_280 + 81_920 + 311_296 + 5_120 + 19_456


def test_profiled_traffic_comes_from_the_committed_summary():
    t = bench.profiled_traffic()
    assert isinstance(t, int)
    # every weight byte crosses HBM once: within 1 % of the algorithmic bytes
    assert abs(t - bench.BYTES_PER_CALL) <= 0.01 * bench.BYTES_PER_CALL


def test_measured_peaks_file_or_fallback(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    assert bench.measured_peaks() == (6650.0, "fallback")
    assert bench.measured_tflops() == (1590.0, 1400.0, "fallback")
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps(
        {"hbm_gbs": 6536.4, "bf16_tflops": 1615.2, "bf16_tflops_sustained": 1402.0}))
    assert bench.measured_peaks() == (6536.4, "measured")
    assert bench.measured_tflops() == (1615.2, 1402.0, "measured")


def test_timeline_summary_of_synthetic_stamps():
    # 4 calls x 3 CTAs, slots 0 (entry) and 1 (exit); call c starts at 10 us * c
    calls, grid = 4, 3
    t = np.zeros((calls, grid, 16), dtype=np.int64)
    for c in range(calls):
        base = 10_000 * (c + 1)
        t[c, :, 0] = base + np.array([0, 1_000, 2_000])     # entries 0 / 1 / 2 us after the first
        t[c, :, 1] = base + np.array([6_000, 7_000, 12_000])  # exits; the last one 12 us in
    out = bench._timeline_summary(t, [(0, "entry"), (1, "exit")], calls)
    assert out["entry"] == 1.0          # median CTA enters 1 us after the call's first entry
    assert out["exit"] == 7.0
    assert out["previous_call_last_exit"] == 2.0   # previous call's last exit (12 us) - 10 us
    assert out["period"] == 10.0


def test_repository_root_is_where_bench_lives():
    assert os.path.samefile(bench.ROOT, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
