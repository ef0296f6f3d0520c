"""Achieved-bandwidth columns for AKO's benchmark reports.

AKO's ``BenchmarkReport`` (reference ``ako/benchmark/report.py:15-80``) records
latencies only. Its sweep runners add one row per kernel and shape with the
first input's shape and the dtype (``ako/benchmark/rmsnorm_bench.py:96``,
``ako/benchmark/rope_bench.py:97``, ``scripts/benchmark_swiglu.py:82``) and one
comparison per candidate (``report.py:30-69``). ``add_bandwidth`` adds, to each
of them, the op's algorithmic bytes and the GB/s they imply, and the fraction of
a given peak, so a report from a B200 reads against its HBM roofline.

Algorithmic bytes count what the op must move once: the inputs read and the
outputs written, with the weight or the RoPE table rows counted once, not per
row (for a ``(B, S, H, D)`` RoPE input, the S table rows of cos and sin).
"""

from __future__ import annotations

import math
from typing import Any, Sequence

ELEMENT_BYTES = {"float32": 4, "float16": 2, "bfloat16": 2}
OPS = ("rmsnorm", "rmsnorm_residual", "rope", "swiglu")


def algorithmic_bytes(op: str, shape: Sequence[int], dtype: str) -> int:
    """Bytes one call of ``op`` moves, for a first input of ``shape`` in ``dtype``.

    rmsnorm: read x, write y (``2 M H b``) plus the weight (``H b``);
    rmsnorm_residual: read x and the residual, write y and the new residual
    (``4 M H b``) plus the weight; rope: read and write x (``2 B S H D b``) plus
    the S fp32 cos and sin rows (``S (D / 2) 4 2``); swiglu: read gate and up,
    write y (``3 M F b``). M is the product of the leading dimensions.
    """
    if dtype not in ELEMENT_BYTES:
        raise ValueError(f"unsupported dtype '{dtype}'")
    b = ELEMENT_BYTES[dtype]
    shape = [int(s) for s in shape]
    if not shape:
        raise ValueError("empty shape")
    last = shape[-1]
    m = math.prod(shape[:-1])
    if op == "rmsnorm":
        return 2 * m * last * b + last * b
    if op == "rmsnorm_residual":
        return 4 * m * last * b + last * b
    if op == "rope":
        if len(shape) != 4:
            raise ValueError(f"rope takes a (batch, seq_len, heads, head_dim) input, got shape {shape}")
        s, d = shape[1], shape[3]
        return 2 * m * last * b + s * (d // 2) * 4 * 2
    if op == "swiglu":
        return 3 * m * last * b
    raise ValueError(f"unknown op '{op}' (expected one of {', '.join(OPS)})")


def _gbs(nbytes: int, ms: float | None) -> float | None:
    return round(nbytes / (ms * 1e-3) / 1e9, 2) if ms else None


def add_bandwidth(report: Any, peak_gbs: float | None = None) -> Any:
    """Add bandwidth columns to an AKO ``BenchmarkReport`` in place and return it.

    Each result row gains ``algorithmic_bytes``, ``achieved_gbs`` (from the
    device time ``gpu_p50_ms`` when the row has one, else the wall-clock
    ``latency_p50_ms``), ``gbs_time`` (which of the two) and, with
    ``peak_gbs``, ``frac_of_peak``. Each comparison gains ``algorithmic_bytes``
    and the GB/s of its candidate, its baseline and, when recorded, its best
    baseline (from their wall-clock p50s, the times a comparison holds).
    Rows without a shape or a known dtype are left as they are.
    """
    op = report.operation
    for row in report.results:
        try:
            nbytes = algorithmic_bytes(op, row["shape"], row["dtype"])
        except (KeyError, ValueError):
            continue
        source = "gpu_p50_ms" if row.get("gpu_p50_ms") else "latency_p50_ms"
        gbs = _gbs(nbytes, row.get(source))
        row["algorithmic_bytes"] = nbytes
        row["achieved_gbs"] = gbs
        row["gbs_time"] = source
        if peak_gbs and gbs is not None:
            row["frac_of_peak"] = round(gbs / peak_gbs, 4)
    for row in report.comparisons:
        try:
            nbytes = algorithmic_bytes(op, row["shape"], row["dtype"])
        except (KeyError, ValueError):
            continue
        row["algorithmic_bytes"] = nbytes
        row["candidate_gbs"] = _gbs(nbytes, row.get("candidate_ms"))
        row["baseline_gbs"] = _gbs(nbytes, row.get("baseline_ms"))
        if row.get("best_baseline_ms") is not None:
            row["best_baseline_gbs"] = _gbs(nbytes, row["best_baseline_ms"])
        if peak_gbs and row["candidate_gbs"] is not None:
            row["candidate_frac_of_peak"] = round(row["candidate_gbs"] / peak_gbs, 4)
    return report


__all__ = ["ELEMENT_BYTES", "OPS", "algorithmic_bytes", "add_bandwidth"]
