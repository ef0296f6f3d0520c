"""CPU tests of the bandwidth columns added to AKO's own benchmark reports:
the per-op algorithmic bytes, and rows filled the way AKO's sweep runners fill
them (a real ``BenchResult`` from AKO's ``bench_op`` on CPU, and comparisons
from ``add_comparison``)."""

from __future__ import annotations

import pytest
import torch

from ako_b200 import bandwidth
from ako_b200.reference import ako


def test_algorithmic_bytes_per_op() -> None:
    # the bench headline cell: 4 x 32768 x 16384 x 2 + 16384 x 2
    assert bandwidth.algorithmic_bytes("rmsnorm_residual", (32768, 16384), "bfloat16") == 4_295_000_064
    # config 1 with leading dims: [4, 512, 4096] fp32
    assert bandwidth.algorithmic_bytes("rmsnorm", (4, 512, 4096), "float32") == 2 * 2048 * 4096 * 4 + 4096 * 4
    # RoPE q at 32 x 4096 x 32 x 128: x read and written, 4096 cos and sin rows of 64 fp32
    assert bandwidth.algorithmic_bytes("rope", (32, 4096, 32, 128), "bfloat16") == 2_149_580_800
    assert bandwidth.algorithmic_bytes("swiglu", (16384, 14336), "bfloat16") == 1_409_286_144
    with pytest.raises(ValueError, match="unknown op"):
        bandwidth.algorithmic_bytes("gelu", (4, 4), "float32")
    with pytest.raises(ValueError, match="dtype"):
        bandwidth.algorithmic_bytes("rmsnorm", (4, 4), "int8")
    with pytest.raises(ValueError, match="head_dim"):
        bandwidth.algorithmic_bytes("rope", (4, 4), "float32")


def test_columns_on_an_ako_report() -> None:
    ako()
    from ako.benchmark.bench_op import bench_op
    from ako.benchmark.report import BenchmarkReport
    from ako.ops.rmsnorm_ref import rmsnorm_ref

    x = torch.randn(2, 8, 64)
    w = torch.ones(64)
    result = bench_op(rmsnorm_ref, (x, w), warmup=1, repeats=2, kernel_name="rmsnorm_ref")
    report = BenchmarkReport(operation="rmsnorm", device=None)
    report.add_result(result, dtype="float32")
    report.results.append({"kernel_name": "fake", "shape": [2, 8, 64], "dtype": "float32",
                           "latency_p50_ms": 1.0, "gpu_p50_ms": 0.5})
    report.results.append({"kernel_name": "no_shape", "dtype": "float32", "latency_p50_ms": 1.0})
    report.add_comparison(shape=[2, 8, 64], baseline_ms=2.0, candidate_ms=0.5, max_error=0.0,
                          selected_kernel="fake", dtype="float32", best_baseline_ms=1.0,
                          best_baseline_kernel="rmsnorm_torch_native")
    out = bandwidth.add_bandwidth(report, peak_gbs=0.01)
    assert out is report
    nbytes = 2 * 16 * 64 * 4 + 64 * 4
    real, fake, bare = report.results
    assert real["algorithmic_bytes"] == nbytes and real["gbs_time"] == "latency_p50_ms"  # CPU: no device time
    assert real["achieved_gbs"] == pytest.approx(nbytes / (real["latency_p50_ms"] * 1e-3) / 1e9, rel=1e-2, abs=0.01)
    assert fake["gbs_time"] == "gpu_p50_ms" and fake["achieved_gbs"] == round(nbytes / 0.5e-3 / 1e9, 2)
    assert fake["frac_of_peak"] == round(fake["achieved_gbs"] / 0.01, 4)
    assert "achieved_gbs" not in bare
    (cmp,) = report.comparisons
    assert cmp["candidate_gbs"] == round(nbytes / 0.5e-3 / 1e9, 2)
    assert cmp["baseline_gbs"] == round(nbytes / 2e-3 / 1e9, 2)
    assert cmp["best_baseline_gbs"] == round(nbytes / 1e-3 / 1e9, 2)
    assert "candidate_frac_of_peak" in cmp
