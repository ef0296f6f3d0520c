"""CPU tests of the measurement tools: the reference arm of ``bench.py`` (AKO's
own reference on the host cores, with the C restatement beside it) keeps the
JSON line contract, ``bench.py`` refuses fewer than 3 warm-up steps, the
global batch's shards are its rows, and the sweep report renders its tables
and counts from a sweep JSON."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from ako_b200.benchmark.sweep import cell_label, report

REPO = Path(__file__).resolve().parents[1]


def _bench(*args: str, timeout: int = 240) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, "bench.py", *args], cwd=REPO, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_json_line() -> None:
    proc = _bench("--impl", "reference", "--steps", "1", "--warmup", "3", "--reference-rows", "1024",
                  "--cpu-seconds", "1")
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, proc.stdout
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference"
    assert rec["metric"] == "achieved HBM GB/s" and rec["unit"] == "GB/s" and rec["higher_is_better"] is True
    assert rec["value"] > 0 and rec["steps"] == 1 and rec["warmup"] == 3 and rec["n_gpus"] == 1
    assert rec["config"]["workload"] == "rmsnorm_residual_bf16_32768x16384"
    cb = rec["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == rec["value"] and cb["sample"]
    assert "rmsnorm_residual_ref" in cb["sample"] and cb["cpu_model"] is not None and cb["torch_threads"] >= 1
    assert rec["c_port"]["kind"] == "port" and rec["c_port"]["value"] > 0
    assert rec["e2e"] == {"value": rec["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_bench_refuses_short_warmup() -> None:
    proc = _bench("--impl", "reference", "--steps", "1", "--warmup", "2", timeout=60)
    assert proc.returncode == 2
    assert "--warmup must be >= 3" in proc.stderr


def _cell(op: str, **kw) -> dict:
    base = {"config": {"rmsnorm": 1, "rmsnorm_residual": 2, "rope": 3, "swiglu": 4}[op], "op": op, "dtype": "bf16",
            "bytes": 1 << 20, "max_error": 0.0, "budget": 0.1, "ulps": 0.5, "parity": True, "ours_us": 10.0,
            "ours_gbs": 100.0, "frac": 0.5, "triton_us": 12.0, "compile_us": 20.0, "eager_us": 40.0}
    base.update(kw)
    return base


def test_sweep_report_tables_and_counts() -> None:
    cells = [
        _cell("rmsnorm", dtype="fp32", rows=2048, hidden=4096, triton_us=9.0, ulps=2.0),
        _cell("rmsnorm_residual", rows=8192, hidden=4096),
        _cell("rmsnorm_residual", rows=1, hidden=4096, decode=True, ours_wall_us=20.0, triton_wall_us=40.0,
              compile_wall_us=50.0, eager_wall_us=60.0, ours_graph_us=2.0, triton_graph_us=1.9,
              compile_graph_us=3.0, eager_graph_us=20.0),
        _cell("rope", batch=32, seq=4096, heads=8, tensor="k", head_dim=128, ulps=0.0),
        _cell("swiglu", rows=2048, hidden=14336, packed=True, parity=False),
    ]
    md = report({"peak_gbs": 6542.7, "reference_package": True, "launches": 20, "blocks": 7, "cells": cells})
    assert "with n = 20; median of 7 such blocks" in md
    assert "1 of 5 cells fail AKO's error budget: swiglu bf16 M2048 F14336 packed." in md
    assert "rope 0 (bit-exact)" in md and "rmsnorm 2," in md
    # config 1: Triton faster (9 us vs 10 us) -> 0/1 and x0.90
    assert "| rmsnorm | 1 | 0/1, x0.90 | 1/1, x2.00 | 1/1, x4.00 |" in md
    # the decode cell is not counted with the throughput cells
    assert "| rmsnorm_residual | 1 | 1/1, x1.20 | 1/1, x2.00 | 1/1, x4.00 |" in md
    for cfg in ("## Config 1", "## Config 2", "## Config 3", "## Config 4", "## Decode cells"):
        assert cfg in md
    assert "| fp32 | M2048 H4096 | 10 | - | 100 | 0.500 | - | 0.90 | 2.00 | 4.00 | 2 |" in md
    # with a time launched like the competitors (no programmatic launch), ratios use it
    md2 = report({"peak_gbs": 6542.7, "reference_package": True, "launches": 20, "blocks": 7,
                  "cells": [_cell("rmsnorm", dtype="fp32", rows=2048, hidden=4096, triton_us=9.0, ours_nopdl_us=12.0,
                                  copy_us=8.0)]})
    assert "| fp32 | M2048 H4096 | 10 | 12 | 100 | 0.500 | 1.25 | 0.75 | 1.67 | 3.33 |" in md2
    assert "at most 1.25x its time" in md2
    assert "- vs triton: wall clock, ours faster on 1 of 1 cells (x2.00); in a graph, ours at or below on 0 of 1" in md


def test_cell_labels() -> None:
    assert cell_label(_cell("rmsnorm_residual", rows=32, hidden=8192)) == "M32 H8192"
    assert cell_label(_cell("rope", batch=8, seq=1, heads=32, tensor="q")) == "B8 S1 q(32h)"
    assert cell_label(_cell("swiglu", rows=64, hidden=5632, packed=False)) == "M64 F5632"


def test_clock_summary_window_and_reasons() -> None:
    from ako_b200.benchmark.clocks import summarize

    # (time, sm MHz, max MHz, watts, utilization %, reason mask)
    samples = [(0.0, 1965.0, 1965.0, 300.0, 100.0, 0x4), (0.5, 1900.0, 1965.0, 310.0, 100.0, 0),
               (0.6, 1920.0, 1965.0, 305.0, 100.0, 0x40), (1.5, 800.0, 1965.0, 50.0, 0.0, 0x1)]
    inside = summarize(samples, (0.4, 0.7), "test")
    assert inside["samples"] == 2 and inside["samples_in_timed_region"] == 2
    assert inside["sm_mhz"] == 1910.0 and inside["reasons"] == ["hw_thermal_slowdown"]
    assert inside["rejecting_reason_seen"] is True
    whole = summarize(samples, None, "test")
    assert whole["samples_under_load"] == 3 and whole["sm_max_mhz"] == 1965.0
    assert whole["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]  # gpu_idle is never reported
    # an empty window falls back to every sample and says so
    empty = summarize(samples, (5.0, 6.0), "test")
    assert empty["samples_in_timed_region"] == 0 and empty["samples"] == 4
    assert summarize([], None)["samples"] == 0


def test_sweep_cells_cover_the_benchmark_grid() -> None:
    from ako_b200.benchmark.sweep import cells

    cs = cells({1, 2, 3, 4})
    by = {c: [x for x in cs if x["config"] == c] for c in (1, 2, 3, 4)}
    assert [len(by[c]) for c in (1, 2, 3, 4)] == [1, 40, 36, 48] and len(cs) == 125
    assert by[1][0]["rows"] == 2048 and by[1][0]["hidden"] == 4096 and by[1][0]["dtype"] == "fp32"
    assert {(c["rows"], c["hidden"]) for c in by[2]} == {(m, h) for m in (1, 32, 512, 8192, 32768)
                                                          for h in (2048, 4096, 8192, 16384)}
    assert all(c["decode"] == (c["rows"] <= 32) for c in by[2])
    assert {(c["batch"], c["seq"], c["heads"]) for c in by[3]} == {(b, s, h) for b in (1, 8, 32)
                                                                     for s in (1, 512, 4096) for h in (32, 8)}
    assert all(c["decode"] == (c["seq"] == 1) and c["head_dim"] == 128 for c in by[3])
    assert {(c["rows"], c["hidden"], c["packed"]) for c in by[4]} == {
        (m, f, p) for m in (1, 64, 2048, 16384) for f in (5632, 11008, 14336) for p in (False, True)}
    assert all(c["decode"] == (c["rows"] <= 64) for c in by[4])


def test_shards_of_the_global_batch_are_its_rows() -> None:
    """Each rank generates only its rows, from seeds indexed by global row
    block, so the shards of any GPU count concatenate to the one-GPU batch."""
    import bench
    from ako_b200.sharding import shard_range

    m, h = 5000, 16
    whole_x, whole_r = bench.global_rows(0, m, h, torch.bfloat16, "cpu", 0)
    for world in (2, 3, 8):
        parts = [bench.global_rows(*shard_range(m, world, r), h, torch.bfloat16, "cpu", 0) for r in range(world)]
        assert torch.equal(torch.cat([p[0] for p in parts]), whole_x)
        assert torch.equal(torch.cat([p[1] for p in parts]), whole_r)
    assert not torch.equal(whole_x[:1024], whole_r[:1024])
    w = bench.weight(h, torch.float32, "cpu", 0)
    assert abs(w.mean().item() - 1.0) < 0.1


@pytest.mark.parametrize("shape, per_block, std", [((24,), 1024, 2.0), ((3, 2, 8), 1, 1.0)],
                         ids=["swiglu-rows", "rope-batch"])
def test_shards_of_other_ops_are_their_batch(shape, per_block, std) -> None:
    """SwiGLU rows and RoPE batch entries are drawn per block of the first
    axis, so every GPU count's shards concatenate to the one-GPU tensor."""
    import bench
    from ako_b200.sharding import shard_range

    m = 2500 if per_block > 1 else 11
    whole = bench.global_blocks(0, m, shape, torch.bfloat16, "cpu", 0, std, per_block)
    for world in (2, 3, 8):
        parts = [bench.global_blocks(*shard_range(m, world, r), shape, torch.bfloat16, "cpu", 0, std, per_block)
                 for r in range(world)]
        assert torch.equal(torch.cat(parts), whole)
    assert abs(whole.float().std().item() - std) < 0.1 * std
    other = bench.global_blocks(0, m, shape, torch.bfloat16, "cpu", 7, std, per_block)
    assert not torch.equal(other, whole)


def test_host_rows_that_fit_is_bounded() -> None:
    import bench

    rows = bench.host_rows_that_fit(32768, 16384, 2)
    assert bench.ROW_BLOCK <= rows <= 32768 and rows % bench.ROW_BLOCK == 0
    desc = bench.cpu_description()
    assert desc["os_cpu_count"] >= 1 and desc["torch_threads"] >= 1
