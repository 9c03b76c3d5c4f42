"""bench.py's plumbing without a GPU: the committed ncu summaries it reads the roofline traffic
from, the peaks it divides by, the shapes it times and its argument rules."""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


@pytest.mark.parametrize("summary", ["w8a8_gemm_sm100_70b_ffn", "q4_0_gemv_70b_decode"])
def test_roofline_traffic_comes_from_the_committed_profile(summary: str) -> None:
    traffic = bench.profile_traffic(summary)
    assert traffic is not None and traffic > 0
    # the traffic is one launch's DRAM bytes: at least the algorithmic bytes of the kernel
    minimum = {"w8a8_gemm_sm100_70b_ffn": 738e6, "q4_0_gemv_70b_decode": 132e6}[summary]
    assert traffic >= minimum


def test_peaks_and_shapes() -> None:
    peaks, kind = bench.measured_peaks()
    assert kind in ("measured", "fallback")
    assert set(peaks) == {"hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"}
    assert all(value > 0 for value in peaks.values())
    assert bench.shapes() == [("gate_proj", 8192, 28672), ("up_proj", 8192, 28672), ("down_proj", 28672, 8192)]


def test_argument_rules() -> None:
    result = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--steps", "1", "--warmup", "1"],
        capture_output=True,
        text=True,
        timeout=120,
        cwd=ROOT,
    )
    assert result.returncode != 0 and "--warmup must be >= 3" in (result.stderr + result.stdout)


def test_exchange_follows_the_gpu_count() -> None:
    assert bench.resolve_exchange("auto", 1) == "fused"
    assert bench.resolve_exchange("auto", 2) == "copy"
    assert bench.resolve_exchange("auto", 4) == "fused"
    assert bench.resolve_exchange("auto", 8) == "fused"
    assert bench.resolve_exchange("nccl", 2) == "nccl"
    assert bench.resolve_exchange("fused", 2) == "fused"


def test_row_quantizer_traffic_comes_from_the_committed_profile() -> None:
    for k in (8192, 28672):
        traffic = bench.profile_traffic("quantize_rows_int8_70b_ffn", f"k{k}")
        assert traffic is not None and traffic > 4096 * k * 4 * 0.9  # at least the fp32 rows read
