"""bench.py's roofline selection (CPU): the grouped-GEMM family is reported
against the HBM copy peak below the ridge point of the measured peaks and
against the bf16 GEMM peak above it, with both figures in the line."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402

PEAKS = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0}


def test_decode_is_hbm_bound():
    r = bench.gemm_roofline(1.0e9, 1.0e10, 0.5, 18, PEAKS, "measured", None)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert abs(r["achieved"] - 2000.0) < 1e-6 and abs(r["frac"] - 2000.0 / 6500.0) < 1e-12
    assert abs(r["achieved_tflops"] - 20.0) < 1e-9


def test_prefill_is_tensor_bound():
    r = bench.gemm_roofline(1.0e9, 1.0e12, 1.0, 18, PEAKS, "measured", 1.8e10)
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert abs(r["achieved"] - 1000.0) < 1e-6 and abs(r["frac"] - 1000.0 / 1600.0) < 1e-12
    assert r["traffic"] == 1.0e9 and r["arithmetic_intensity"] > r["ridge"]
