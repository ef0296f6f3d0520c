"""Per-cell sweep of the four benchmark configurations on one GPU, with competitors.

For every op / shape / dtype cell it reports the device time of the sm_100a
kernel from a cold L2 (differential timing: n x (2x-L2 read, call) minus n
reads, over n; event steps of ~2 us average out and each call is charged
the write-back of its outputs), the achieved GB/s on the algorithmic bytes,
and the fraction of the measured HBM copy bandwidth. Competitors come from the
reference package and are timed the same way: AKO's unfused reference
(eager), its ``torch.compile`` form, ``F.rms_norm`` and AKO's own Triton
kernels. Ours is timed twice: as shipped (programmatic dependent launch on,
which lets a call's launch overlap the end of the flush read before it), and
through the measurement build with programmatic launch off, launched like the
competitors; the kernel-to-kernel comparison uses the second. Decode cells
(one token per sequence) add the wall-clock latency per call of back-to-back
calls, which is what a decode loop pays, and the device time per call of 20
calls captured in one CUDA graph. Each cell is also checked against AKO's
eager reference with AKO's error budget, and timed against a plain
device-to-device copy of its algorithmic bytes (half read, half written),
timed the same way: the practical roofline at that size, since ramp-up, the
last wave and the final write-back cost a fixed few microseconds.

    python -m ako_b200.benchmark.sweep --out sweep.json [--configs 1,2,3,4]
    python -m ako_b200.benchmark.sweep --report sweep.json > sweep.md

``--report`` renders a sweep JSON as markdown tables with summary counts.
"""

from __future__ import annotations

import argparse
import json
import math
import statistics
import time
from pathlib import Path
from typing import Any, Callable

import torch

from ako_b200 import _native, kernels
from ako_b200.benchmark.timing import Flusher, cold_us
from ako_b200.reference import ako

DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}


def _reference_package():
    ako()
    from ako.ops import rmsnorm_ref, rmsnorm_torch, rmsnorm_triton, rope_ref, rope_torch, rope_triton, swiglu_ref
    from ako.ops import swiglu_torch, swiglu_triton

    return {
        "rmsnorm": {"eager": rmsnorm_ref.rmsnorm_ref, "compile": rmsnorm_torch.rmsnorm_compiled,
                    "triton": rmsnorm_triton.rmsnorm_triton},
        "rmsnorm_residual": {"eager": rmsnorm_ref.rmsnorm_residual_ref,
                             "compile": rmsnorm_torch.rmsnorm_residual_compiled,
                             "triton": rmsnorm_triton.rmsnorm_residual_triton},
        "rope": {"eager": rope_ref.rope_ref, "compile": rope_torch.rope_compiled, "triton": rope_triton.rope_triton},
        "swiglu": {"eager": swiglu_ref.swiglu_ref, "compile": swiglu_torch.swiglu_compiled,
                   "triton": swiglu_triton.swiglu_triton},
    }


OURS = {
    "rmsnorm": kernels.rmsnorm_cuda_sm100,
    "rmsnorm_residual": kernels.rmsnorm_residual_cuda_sm100,
    "rope": kernels.rope_cuda_sm100,
    "swiglu": kernels.swiglu_cuda_sm100,
}


def cells(configs: set[int]) -> list[dict[str, Any]]:
    out: list[dict[str, Any]] = []
    if 1 in configs:
        out.append({"config": 1, "op": "rmsnorm", "dtype": "fp32", "rows": 2048, "hidden": 4096, "eps": 1e-6})
    if 2 in configs:
        for dt in ("bf16", "fp16"):
            for h in (2048, 4096, 8192, 16384):
                for m in (1, 32, 512, 8192, 32768):
                    out.append({"config": 2, "op": "rmsnorm_residual", "dtype": dt, "rows": m, "hidden": h,
                                "eps": 1e-5, "decode": m <= 32})
    if 3 in configs:
        for dt in ("bf16", "fp16"):
            for b in (1, 8, 32):
                for s in (1, 512, 4096):
                    for heads, which in ((32, "q"), (8, "k")):
                        out.append({"config": 3, "op": "rope", "dtype": dt, "batch": b, "seq": s, "heads": heads,
                                    "tensor": which, "head_dim": 128, "decode": s == 1})
    if 4 in configs:
        for dt in ("bf16", "fp16"):
            for f in (5632, 11008, 14336):
                for m in (1, 64, 2048, 16384):
                    for packed in (False, True):
                        out.append({"config": 4, "op": "swiglu", "dtype": dt, "rows": m, "hidden": f,
                                    "packed": packed, "decode": m <= 64})
    return out


def make_inputs(cell: dict[str, Any], dev: torch.device, tables: dict) -> tuple[tuple, dict, int]:
    """Seeded inputs, call kwargs and algorithmic bytes of one cell."""
    dt = DTYPES[cell["dtype"]]
    b = torch.tensor([], dtype=dt).element_size()
    g = torch.Generator(device=dev).manual_seed(0)
    rnd = lambda *s, m=0.0, sd=1.0: (torch.randn(*s, generator=g, device=dev) * sd + m).to(dt)  # noqa: E731
    op = cell["op"]
    if op in ("rmsnorm", "rmsnorm_residual"):
        m, h = cell["rows"], cell["hidden"]
        x, w = rnd(m, h), rnd(h, m=1.0, sd=0.1)
        if op == "rmsnorm":
            return (x, w, cell["eps"]), {}, 2 * m * h * b + h * b
        return (x, rnd(m, h), w, cell["eps"]), {}, 4 * m * h * b + h * b
    if op == "rope":
        bb, s, hh, d = cell["batch"], cell["seq"], cell["heads"], cell["head_dim"]
        cos_full, sin_full = tables[d]
        off = 2047 if s == 1 else 0
        x = rnd(bb, s, hh, d)
        return (x, cos_full[off:off + s], sin_full[off:off + s], "neox"), {}, 2 * x.numel() * b + s * (d // 2) * 8
    m, f = cell["rows"], cell["hidden"]
    if cell["packed"]:
        p = rnd(m, 2 * f, sd=2.0)
        return (p[:, :f], p[:, f:]), {}, 3 * m * f * b
    return (rnd(m, f, sd=2.0), rnd(m, f, sd=2.0)), {}, 3 * m * f * b


def device_us(fn: Callable, args: tuple, n: int, flush: Flusher, blocks: int) -> float:
    """Cold-L2 device time of one call (differential timing, see ako_b200.benchmark.timing)."""
    return cold_us(lambda: fn(*args), flush, n=n, blocks=blocks)


def wall_us(fn: Callable, args: tuple, batches: int = 15, inner: int = 50) -> float:
    """Wall-clock per call of back-to-back calls (p50 over batches)."""
    for _ in range(5):
        fn(*args)
    torch.cuda.synchronize()
    samples = []
    for _ in range(batches):
        t0 = time.perf_counter()
        for _ in range(inner):
            fn(*args)
        torch.cuda.synchronize()
        samples.append((time.perf_counter() - t0) * 1e6 / inner)
    return statistics.median(samples)


def graph_us(fn: Callable, args: tuple, calls: int = 20, replays: int = 40) -> float | None:
    """Device time per call of ``calls`` calls captured in one CUDA graph (best
    of three timed runs of ``replays`` replays); None if capture fails."""
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn(*args)
        torch.cuda.current_stream().wait_stream(side)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for _ in range(calls):
                fn(*args)
        for _ in range(2):
            gr.replay()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(3):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(replays):
                gr.replay()
            e.record()
            torch.cuda.synchronize()
            best = min(best, s.elapsed_time(e) * 1e3 / (replays * calls))
        return round(best, 3)
    except Exception:  # noqa: BLE001 - a candidate that cannot be captured is reported as such
        return None


# ------------------------------------------------------------------ report
TITLES = {
    1: "Config 1 — RMSNorm fp32 [4,512,4096] (2048 rows x 4096)",
    2: "Config 2 — fused residual-add RMSNorm",
    3: "Config 3 — RoPE neox, D=128, fp32 [8192,64] table sliced (S=1 at position 2047)",
    4: "Config 4 — SwiGLU, separate [M,F] or packed [M,2F]",
}
COMPETITORS = ("triton", "compile", "eager")


def cell_label(c: dict[str, Any]) -> str:
    if c["op"] in ("rmsnorm", "rmsnorm_residual"):
        return f"M{c['rows']} H{c['hidden']}"
    if c["op"] == "rope":
        return f"B{c['batch']} S{c['seq']} {c['tensor']}({c['heads']}h)"
    return f"M{c['rows']} F{c['hidden']}" + (" packed" if c.get("packed") else "")


def _fmt(v: float | None, nd: int = 3) -> str:
    if v is None:
        return "-"
    return f"{v:.{nd}g}" if v < 100 else f"{v:.0f}" if v >= 1000 else f"{v:.1f}"


def _ratio(c: dict[str, Any], name: str, key: str = "us") -> float | None:
    """Competitor time over ours; device times compare with ours launched like them (no PDL)."""
    theirs = c.get(f"{name}_{key}")
    ours = c.get("ours_nopdl_us", c.get("ours_us")) if key == "us" else c.get(f"ours_{key}")
    return theirs / ours if theirs and ours else None


def _geomean(xs: list[float]) -> float:
    return math.exp(sum(math.log(x) for x in xs) / len(xs)) if xs else float("nan")


def report(summary: dict[str, Any]) -> str:
    """Markdown tables and summary counts of one sweep JSON."""
    cells = summary["cells"]
    peak = summary["peak_gbs"]
    n, blocks = summary.get("launches", 20), summary.get("blocks", 5)
    out = ["# Per-cell sweep of benchmark configurations 1-4 on one B200", "",
           "    python -m ako_b200.benchmark.sweep --out sweep.json",
           "    python -m ako_b200.benchmark.sweep --report sweep.json", "",
           "Columns:",
           f"- `us`: device time of one call from a cold L2, differential: n x (read of 2 x the L2 size, call)",
           f"  minus n reads, over n, with n = {n}; median of {blocks} such blocks. The read evicts the previous",
           "  call's outputs, so each call is charged the write-back of what it wrote.",
           f"- `GB/s`: algorithmic bytes over `us`. `frac`: that over the measured {peak} GB/s copy bandwidth.",
           "- Competitors are timed the same way:",
           "  - `triton`: AKO's own Triton kernels, JIT-compiled for sm_100 on this GPU;",
           "  - `compile`: AKO's `torch.compile` form of the reference;",
           "  - `eager`: AKO's unfused reference.",
           "  All three come from the reference package (installed offline into `baseline/_ref`).",
           "- `us nopdl`: ours through the measurement build with programmatic dependent launch off, launched",
           "  like the competitors. `x` columns and the summary compare each competitor with it (above 1: ours",
           "  is faster); `us` is ours as shipped (programmatic launch on).",
           "- `ulps`: AKO's `error_in_ulps` of our output against its eager reference.",
           "- `copy`: a plain device-to-device copy of the cell's algorithmic bytes, timed the same way; `us/copy` is",
           "  ours (as shipped) over it: the practical roofline at that size.", ""]
    fails = [c for c in cells if not c["parity"]]
    out.append(f"All {len(cells)} cells pass AKO's error budget." if not fails else
               f"{len(fails)} of {len(cells)} cells fail AKO's error budget: " +
               ", ".join(f"{c['op']} {c['dtype']} {cell_label(c)}" for c in fails) + ".")
    maxu = {}
    for c in cells:
        maxu[c["op"]] = max(maxu.get(c["op"], 0.0), c["ulps"])
    out.append("Max reported ulps: " + ", ".join(f"{op} {u:g}" + (" (bit-exact)" if u == 0 else "")
                                                 for op, u in maxu.items()) + ".")
    vs_copy = [c["ours_us"] / c["copy_us"] for c in cells if c.get("copy_us") and not c.get("decode")]
    if vs_copy:
        out.append(f"Throughput cells against a copy of the same bytes: at most {max(vs_copy):.2f}x its time, "
                   f"geometric mean {_geomean(vs_copy):.2f}x.")
    out.append("")
    out.append("Throughput cells (not decode), ours against each competitor: cells where ours is at or below "
               "its time, and the geometric mean of its time over ours.")
    out.append("")
    out.append("| op | cells | " + " | ".join(f"vs {n}" for n in COMPETITORS) + " |")
    out.append("|---|---:|" + "---|" * len(COMPETITORS))
    for op in dict.fromkeys(c["op"] for c in cells):
        cs = [c for c in cells if c["op"] == op and not c.get("decode")]
        if not cs:
            continue
        parts = []
        for n in COMPETITORS:
            rs = [r for r in (_ratio(c, n) for c in cs) if r]
            parts.append(f"{sum(r >= 1.0 for r in rs)}/{len(rs)}, x{_geomean(rs):.2f}" if rs else "-")
        out.append(f"| {op} | {len(cs)} | " + " | ".join(parts) + " |")
    out.append("")
    for cfg in sorted({c["config"] for c in cells}):
        out += [f"## {TITLES[cfg]}", "",
                "| dtype | cell | us | us nopdl | GB/s | frac | us/copy | " + " | ".join(f"x {n}" for n in COMPETITORS)
                + " | ulps |",
                "|---|---|---:|---:|---:|---:|---:|" + "---:|" * len(COMPETITORS) + "---:|"]
        for c in cells:
            if c["config"] != cfg:
                continue
            xs = " | ".join(f"{r:.2f}" if (r := _ratio(c, n)) else "-" for n in COMPETITORS)
            vc = f"{c['ours_us'] / c['copy_us']:.2f}" if c.get("copy_us") else "-"
            out.append(f"| {c['dtype']} | {cell_label(c)} | {_fmt(c['ours_us'])} | {_fmt(c.get('ours_nopdl_us'))} | "
                       f"{c['ours_gbs']:.0f} | {c['frac']:.3f} | {vc} | {xs} | {c['ulps']:g} |")
        out.append("")
    dec = [c for c in cells if c.get("decode")]
    if dec:
        out += ["## Decode cells: latency a decode loop pays", "",
                "- `wall`: wall clock per call of back-to-back calls from Python (p50 of 15 batches of 50). This is",
                "  what AKO's selector compares (`latency_p50_ms`).",
                "- `graph`: device time per call of 20 calls captured in one CUDA graph (best of 3 timed runs of",
                "  40 replays).", "",
                "| op | dtype | cell | " + " | ".join(f"wall {n}" for n in ("ours", *COMPETITORS)) + " | " +
                " | ".join(f"graph {n}" for n in ("ours", *COMPETITORS)) + " |",
                "|---|---|---|" + "---:|" * (2 * (1 + len(COMPETITORS)))]
        for c in dec:
            walls = " | ".join(_fmt(c.get(f"{n}_wall_us")) for n in ("ours", *COMPETITORS))
            graphs = " | ".join(_fmt(c.get(f"{n}_graph_us")) for n in ("ours", *COMPETITORS))
            out.append(f"| {c['op']} | {c['dtype']} | {cell_label(c)} | {walls} | {graphs} |")
        out.append("")
        for n in COMPETITORS:
            w = [r for r in (_ratio(c, n, "wall_us") for c in dec) if r]
            g = [r for r in (_ratio(c, n, "graph_us") for c in dec) if r]
            if w or g:
                out.append(f"- vs {n}: wall clock, ours faster on {sum(r > 1 for r in w)} of {len(w)} cells "
                           f"(x{_geomean(w):.2f}); in a graph, ours at or below on {sum(r >= 1 for r in g)} of "
                           f"{len(g)} (x{_geomean(g):.2f}).")
        out.append("")
    return "\n".join(out)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--report", default=None, help="render this sweep JSON as markdown and exit")
    ap.add_argument("--configs", default="1,2,3,4")
    ap.add_argument("--competitors", default="eager,compile,triton,native")
    ap.add_argument("--launches", type=int, default=20, help="calls per timed block")
    ap.add_argument("--blocks", type=int, default=7, help="timed blocks per cell (median)")
    ap.add_argument("--peak-gbs", type=float, default=None)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    if args.report:
        print(report(json.loads(Path(args.report).read_text())))
        return

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak = args.peak_gbs
    if peak is None:
        try:
            peak = float(json.loads(Path("MEASURED_PEAKS.json").read_text())["hbm_gbs"])
        except (OSError, KeyError, ValueError):
            peak = 6650.0
    comps = _reference_package()
    from ako.ops.rmsnorm_torch import rmsnorm_torch_native
    from ako.ops.rope_ref import build_rope_tables
    from ako.validation.numerical import error_budget, error_in_ulps, max_abs_error_any

    wanted = set(args.competitors.split(","))
    flush = Flusher(dev)
    tables = {128: build_rope_tables(8192, 128, device=dev)}
    results = []
    for cell in cells({int(c) for c in args.configs.split(",")}):
        inputs, kw, nbytes = make_inputs(cell, dev, tables)
        op = cell["op"]
        row: dict[str, Any] = {**cell, "bytes": nbytes}
        ours = OURS[op]
        out = ours(*inputs)
        ref = comps[op]["eager"](*inputs)
        row["max_error"] = max_abs_error_any(ref, out)
        row["budget"] = error_budget(ref)
        row["ulps"] = round(error_in_ulps(ref, out), 3)
        row["parity"] = row["max_error"] <= row["budget"]
        us = device_us(ours, inputs, args.launches, flush, args.blocks)
        row["ours_us"] = round(us, 3)
        row["ours_gbs"] = round(nbytes / us / 1e3, 1)
        row["frac"] = round(nbytes / us / 1e3 / peak, 4)
        half = max(16, nbytes // 2)
        src = torch.empty(half, dtype=torch.uint8, device=dev)
        dst = torch.empty_like(src)
        row["copy_us"] = round(device_us(dst.copy_, (src,), args.launches, flush, args.blocks), 3)
        del src, dst
        with _native.measurement() as mlib:
            mlib.ako_b200_set_pdl(0)
            try:
                row["ours_nopdl_us"] = round(device_us(ours, inputs, args.launches, flush, args.blocks), 3)
            finally:
                mlib.ako_b200_set_pdl(1)
        candidates = {k: v for k, v in comps[op].items() if k in wanted}
        if op == "rmsnorm" and "native" in wanted:
            candidates["native"] = rmsnorm_torch_native
        for name, fn in candidates.items():
            try:
                row[f"{name}_us"] = round(device_us(fn, inputs, args.launches, flush, args.blocks), 3)
            except Exception as exc:  # noqa: BLE001 - a competitor that cannot run this cell
                row[f"{name}_us"] = None
                row[f"{name}_error"] = f"{type(exc).__name__}: {str(exc)[:120]}"
        if cell.get("decode"):
            row["ours_wall_us"] = round(wall_us(ours, inputs), 2)
            row["ours_graph_us"] = graph_us(ours, inputs)
            for name, fn in candidates.items():
                if row.get(f"{name}_us") is not None:
                    row[f"{name}_wall_us"] = round(wall_us(fn, inputs), 2)
                    row[f"{name}_graph_us"] = graph_us(fn, inputs)
        results.append(row)
        print(json.dumps(row), flush=True)
        del inputs, out, ref
    summary = {"peak_gbs": peak, "reference_package": True, "launches": args.launches,
               "blocks": args.blocks,
               "gpu": torch.cuda.get_device_name(dev), "cells": results}
    if args.out:
        Path(args.out).write_text(json.dumps(summary, indent=1))


if __name__ == "__main__":
    main()
