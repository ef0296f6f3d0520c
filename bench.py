#!/usr/bin/env python
"""Benchmark of the B200 kernels behind AKO's dispatcher API; prints ONE JSON line.

Metric: achieved HBM GB/s = algorithmic bytes / device time (the first half
of the reference configuration's metric; the decoder's prefill and decode
tokens per second, the second half, are in ``decoder``).

A step is one pass of the hot path over one batch: by default one fused
residual-add RMSNorm (``rmsnorm_residual``) over config 2's largest cell,
32768 rows x 16384 bf16 (4.3 GB moved, far above the 126 MB L2, so
back-to-back steps need no flush).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one process per GPU): the step's batch is one global
batch whose rows (batch entries for the RoPE workloads) are split into
contiguous blocks by ``ako_b200.sharding.shard_range`` (strong scaling;
``--scaling weak`` gives every rank a whole batch instead). Every rank
generates only its own rows, from seeds that depend on the global row index,
so the union of the shards is the one-GPU batch. No collective touches the data path: only a barrier, the
max of the per-rank device times and the AND of the per-rank parity checks.

* ``value``: whole-job GB/s = the global batch's bytes / the slowest rank's
  time, inputs resident in HBM, CUDA events on the launching stream around
  exactly K steps.
* ``weak`` (N > 1): the same with a whole batch per rank.
* ``parity``: every shard against the C oracle: for RMSNorm every row against
  the C model of the kernels' fixed summation order (bit for bit) and three
  rows against the reference-order oracle (the gate); every batch entry of
  RoPE bit for bit; every row of SwiGLU within 2 ulp.
* ``e2e``: the same metric through the host-buffer call
  (``ako_b200.host.rmsnorm_residual_host``): pinned host inputs copied in and
  results copied out inside the timed region, every step.
* ``roofline``: this rank's kernel bytes per launch / its launch time against
  the measured HBM copy bandwidth (``MEASURED_PEAKS.json``), with the DRAM
  traffic of one launch from the committed ncu summary of this workload.
* ``cpu_baseline``: AKO's own unfused reference (``ako.ops.rmsnorm_ref.
  rmsnorm_residual_ref``) on CPU tensors, timed with AKO's ``bench_op``, on
  rows of the same workload, with the CPU described; the C restatement of it
  (``oracle/``, all host threads) as a second number. Rank 0, N = 1.
* ``ops``: the other ops at their largest benchmark cells (N = 1), device time
  per call from a cold L2 (differential timing).
* ``decoder``: configuration 5 (N = 1): prefill and decode tokens per second
  of the B200 decoder (eager and one CUDA graph per step) next to the same
  stack on the reference math, and AKO's own decoder stack through AKO's
  selector with and without the sm_100a candidates.

``--impl reference`` times AKO's own reference (``rmsnorm_residual_ref`` on
CPU tensors, through ``bench_op``) on rank 0 over the workload's rows that the
host memory holds, and prints the same line with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import re
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
NOMINAL_HBM_GBS = 8000.0  # B200 HBM3e datasheet figure, the metric's "% of ~8 TB/s"
ROW_BLOCK = 1024  # rows generated from one seed; shards start on these boundaries when they can

WORKLOADS = {
    # name: (op, dims, dtype)
    "rmsnorm_residual_bf16_32768x16384": ("rmsnorm_residual", (32768, 16384), torch.bfloat16),
    "rmsnorm_residual_bf16_32768x4096": ("rmsnorm_residual", (32768, 4096), torch.bfloat16),
    "rmsnorm_residual_bf16_8192x4096": ("rmsnorm_residual", (8192, 4096), torch.bfloat16),
    "rmsnorm_residual_bf16_4096x8192": ("rmsnorm_residual", (4096, 8192), torch.bfloat16),
    "rmsnorm_fp32_2048x4096": ("rmsnorm", (2048, 4096), torch.float32),
    "rmsnorm_bf16_8192x65536": ("rmsnorm", (8192, 65536), torch.bfloat16),
    "rmsnorm_bf16_8192x32768": ("rmsnorm", (8192, 32768), torch.bfloat16),
    "rope_q_bf16_32x4096x32x128": ("rope", (32, 4096, 32, 128), torch.bfloat16),
    "rope_k_bf16_32x4096x8x128": ("rope", (32, 4096, 8, 128), torch.bfloat16),
    "rope_qk_bf16_32x4096x32+8x128": ("rope_qk", (32, 4096, 32, 128), torch.bfloat16),
    "rope_q_bf16_8x512x32x128": ("rope", (8, 512, 32, 128), torch.bfloat16),
    "swiglu_bf16_16384x14336": ("swiglu", (16384, 14336), torch.bfloat16),
    "swiglu_packed_bf16_16384x14336": ("swiglu_packed", (16384, 14336), torch.bfloat16),
    "swiglu_bf16_2048x14336": ("swiglu", (2048, 14336), torch.bfloat16),
    "swiglu_packed_bf16_2048x14336": ("swiglu_packed", (2048, 14336), torch.bfloat16),
    # small cases of the same kernels (a few hundred MB, above L2) for ncu captures
    "rmsnorm_residual_bf16_2048x16384": ("rmsnorm_residual", (2048, 16384), torch.bfloat16),
    "rmsnorm_residual_bf16_4096x4096": ("rmsnorm_residual", (4096, 4096), torch.bfloat16),
    "rmsnorm_bf16_1024x65536": ("rmsnorm", (1024, 65536), torch.bfloat16),   # chunked persistent kernel
    "rmsnorm_bf16_1024x32768": ("rmsnorm", (1024, 32768), torch.bfloat16),   # staged persistent kernel
    "rmsnorm_bf16_16384x4100": ("rmsnorm", (16384, 4100), torch.bfloat16),   # any-width kernel (8200-byte rows)
    "rope_q_bf16_16x512x32x100": ("rope", (16, 512, 32, 100), torch.bfloat16),  # 4-byte accesses
    "rope_q_bf16_16x512x32x98": ("rope", (16, 512, 32, 98), torch.bfloat16),    # one pair per thread
    "rope_q_bf16_16x512x32x128": ("rope", (16, 512, 32, 128), torch.bfloat16),
    "rope_qk_bf16_8x512x32+8x128": ("rope_qk", (8, 512, 32, 128), torch.bfloat16),
}
DEFAULT_WORKLOAD = "rmsnorm_residual_bf16_32768x16384"
OPS_EXTRA = [
    "rmsnorm_fp32_2048x4096",
    "rmsnorm_residual_bf16_32768x4096",
    "rope_q_bf16_32x4096x32x128",
    "rope_k_bf16_32x4096x8x128",
    "rope_qk_bf16_32x4096x32+8x128",
    "swiglu_bf16_16384x14336",
    "swiglu_packed_bf16_16384x14336",
]


def log(*a: object) -> None:
    print(*a, file=sys.stderr, flush=True)


# ----------------------------------------------------------------- workloads
def row_block(block: int, hidden: int, dtype: torch.dtype, device, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Rows ``[block * ROW_BLOCK, (block + 1) * ROW_BLOCK)`` of x and residual
    of the seeded global batch (N(0, 1)), the same on every rank and GPU count."""
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + block)
    x = torch.randn(ROW_BLOCK, hidden, generator=g, device=device).to(dtype)
    r = torch.randn(ROW_BLOCK, hidden, generator=g, device=device).to(dtype)
    return x, r


def global_rows(lo: int, hi: int, hidden: int, dtype: torch.dtype, device, seed: int):
    """Rows ``[lo, hi)`` of x and residual of the seeded global batch."""
    x = torch.empty(hi - lo, hidden, dtype=dtype, device=device)
    r = torch.empty_like(x)
    for b in range(lo // ROW_BLOCK, (hi + ROW_BLOCK - 1) // ROW_BLOCK):
        bx, br = row_block(b, hidden, dtype, device, seed)
        a, z = max(lo, b * ROW_BLOCK), min(hi, (b + 1) * ROW_BLOCK)
        x[a - lo:z - lo] = bx[a - b * ROW_BLOCK:z - b * ROW_BLOCK]
        r[a - lo:z - lo] = br[a - b * ROW_BLOCK:z - b * ROW_BLOCK]
    return x, r


def global_blocks(lo: int, hi: int, shape: tuple[int, ...], dtype: torch.dtype, device, seed: int, std: float,
                  per_block: int) -> torch.Tensor:
    """Entries ``[lo, hi)`` along the first axis of a seeded N(0, std) tensor
    of entries ``shape``, drawn ``per_block`` entries per seed, so a shard's
    bytes do not depend on how the batch is split."""
    out = torch.empty(hi - lo, *shape, dtype=dtype, device=device)
    for b in range(lo // per_block, (hi + per_block - 1) // per_block):
        g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + 500_000 + b)
        blk = (torch.randn(per_block, *shape, generator=g, device=device) * std).to(dtype)
        a, z = max(lo, b * per_block), min(hi, (b + 1) * per_block)
        out[a - lo:z - lo] = blk[a - b * per_block:z - b * per_block]
    return out


def weight(hidden: int, dtype: torch.dtype, device, seed: int) -> torch.Tensor:
    """The workload's weight, N(1, 0.1), from a seed no row block uses."""
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + 1_000_000)
    return (torch.randn(hidden, generator=g, device=device) * 0.1 + 1.0).to(dtype)


class Workload:
    """Inputs in HBM, one kernel launch per step, and its algorithmic bytes.

    Each op holds entries ``[lo, hi)`` along the first axis of its seeded
    global batch (rows; the batch for RoPE), the whole batch by default.
    """

    def __init__(self, name: str, device: torch.device, seed: int = 0, rows: tuple[int, int] | None = None) -> None:
        from ako_b200 import kernels

        self.name = name
        self.op, self.dims, self.dtype = WORKLOADS[name]
        b = torch.tensor([], dtype=self.dtype).element_size()
        self.element_size = b
        self.lo, self.hi = rows or (0, self.dims[0])
        n = self.hi - self.lo
        if self.op in ("rmsnorm", "rmsnorm_residual"):
            h = self.dims[1]
            self.x, r = global_rows(self.lo, self.hi, h, self.dtype, device, seed)
            self.w = weight(h, self.dtype, device, seed)
            if self.op == "rmsnorm":
                del r
                self.bytes = 2 * n * h * b + h * b
                self.fn = lambda: kernels.rmsnorm_cuda_sm100(self.x, self.w, 1e-6)
            else:
                self.r = r
                self.bytes = 4 * n * h * b + h * b
                self.fn = lambda: kernels.rmsnorm_residual_cuda_sm100(self.x, self.r, self.w, 1e-5)
            self.desc = {"rows": n, "hidden": h}
            self.kernel = "ako_b200::rms_rows_kernel"
            return
        if self.op in ("rope", "rope_qk"):
            _, s, hh, d = self.dims
            from ako_b200.api import build_rope_tables

            cos, sin = build_rope_tables(8192, d, device=device)
            self.cos, self.sin = cos[:s], sin[:s]
            # one batch entry per seed: q from one seed range, k from another
            self.x = global_blocks(self.lo, self.hi, (s, hh, d), self.dtype, device, seed, 1.0, 1)
            table = s * (d // 2) * 4 * 2
            if self.op == "rope":
                self.bytes = 2 * n * s * hh * d * b + table
                self.fn = lambda: kernels.rope_cuda_sm100(self.x, self.cos, self.sin, "neox")
                self.desc = {"batch": n, "seq": s, "heads": hh, "head_dim": d, "style": "neox",
                             "table": "fp32 [8192, 64] sliced"}
            else:
                self.k = global_blocks(self.lo, self.hi, (s, 8, d), self.dtype, device, seed + 7, 1.0, 1)
                self.bytes = 2 * n * s * (hh + 8) * d * b + table
                self.fn = lambda: kernels.rope_qk_cuda_sm100(self.x, self.k, self.cos, self.sin, "neox")
                self.desc = {"batch": n, "seq": s, "q_heads": hh, "k_heads": 8, "head_dim": d, "style": "neox",
                             "table": "fp32 [8192, 64] sliced, read once for q and k"}
            self.kernel = "ako_b200::rope_vec_kernel"
            return
        f = self.dims[1]
        if self.op == "swiglu_packed":
            self.packed = global_blocks(self.lo, self.hi, (2 * f,), self.dtype, device, seed, 2.0, ROW_BLOCK)
            self.g, self.u = self.packed[:, :f], self.packed[:, f:]
        else:
            self.g = global_blocks(self.lo, self.hi, (f,), self.dtype, device, seed, 2.0, ROW_BLOCK)
            self.u = global_blocks(self.lo, self.hi, (f,), self.dtype, device, seed + 7, 2.0, ROW_BLOCK)
        self.bytes = 3 * n * f * b
        self.fn = lambda: kernels.swiglu_cuda_sm100(self.g, self.u)
        self.desc = {"rows": n, "hidden": f, "packed": self.op == "swiglu_packed"}
        self.kernel = "ako_b200::swiglu_kernel"

    def step(self) -> None:
        self.fn()


# -------------------------------------------------------------- distributed
def dist_setup() -> tuple[int, int, int]:
    from ako_b200 import sharding

    world, rank, local = sharding.env_world()
    torch.cuda.set_device(local)
    if world > 1:
        # NCCL prints its version banner on stdout (fd 1) when a communicator
        # comes up; point fd 1 at stderr until then, so the only line rank 0
        # writes to stdout is the JSON result.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            sharding.init("nccl", timeout_s=300.0, device=torch.device("cuda", local))
            sharding.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    return world, rank, local


def timed_region(step, k: int, w: int, marks=None) -> float:
    """W untimed steps, then exactly K steps between events on the launching
    stream, with a barrier and a synchronize on both sides; ms on this rank.
    ``marks`` (a clock sampler) gets the host times around the timed steps."""
    from ako_b200 import sharding

    for _ in range(w):
        step()
    torch.cuda.synchronize()
    sharding.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if marks is not None:
        marks.mark_start()
    start.record()
    for _ in range(k):
        step()
    end.record()
    torch.cuda.synchronize()
    if marks is not None:
        marks.mark_end()
    sharding.barrier()
    return start.elapsed_time(end)


# ------------------------------------------------------------------- peaks
def hbm_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    try:
        v = float(json.loads(p.read_text())["hbm_gbs"])
        return v, "measured (MEASURED_PEAKS.json hbm_gbs, copy bandwidth)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback 6650 GB/s (earlier measurement on this pool)"


def ncu_traffic(workload: str) -> int | None:
    """DRAM bytes per launch recorded in the committed ncu summary of the workload."""
    p = REPO / "profiles" / f"{workload}.md"
    if not p.exists():
        return None
    m = re.search(r"^traffic_bytes_per_launch:\s*(\d+)", p.read_text(), re.M)
    return int(m.group(1)) if m else None


# ------------------------------------------------------------------ parity
def shard_parity(wl: Workload, threads: int | None = None) -> dict:
    """This rank's shard on the host against the C oracle: three of its rows
    (its first, middle and last; for RoPE, those batch entries). RMSNorm rows
    are held to the C model of the kernels' fixed summation order bit for bit
    and to the reference-order oracle within AKO's ulp bound; RoPE is
    bit-exact; SwiGLU is within 2 ulp (16-bit) of the reference's formula."""
    import numpy as np

    from oracle import ako_oracle as O
    from oracle import c_oracle as C

    def host(t: torch.Tensor) -> np.ndarray:
        t = t.detach().cpu().contiguous()
        return t.view(torch.int16).numpy().view(np.uint16) if t.dtype in (torch.bfloat16, torch.float16) else t.numpy()

    n = wl.hi - wl.lo
    sel = sorted({0, n // 2, n - 1})
    dt = {torch.bfloat16: O.BF16, torch.float16: O.F16, torch.float32: O.F32}[wl.dtype]
    ok, worst = True, 0
    if wl.op in ("rope", "rope_qk"):
        # every batch entry of the shard, bit for bit
        cos, sin = wl.cos.cpu().numpy(), wl.sin.cpu().numpy()
        outs = wl.fn()
        pairs = [(wl.x, outs)] if wl.op == "rope" else [(wl.x, outs[0]), (wl.k, outs[1])]
        for src, out in pairs:
            d = O.ulp_distance(C.rope(host(src), cos, sin, "neox", dt, threads=threads), host(out), dt)
            worst = max(worst, int(d.max()))
        return {"ok": worst == 0, "batch_entries_checked": n, "max_ulp_vs_reference": worst}
    if wl.op in ("swiglu", "swiglu_packed"):
        # every row of the shard
        y = host(wl.fn())
        worst = int(O.ulp_distance(C.swiglu(host(wl.g), host(wl.u), dt, threads=threads), y, dt).max())
        return {"ok": worst <= (2 if dt != O.F32 else 6), "rows_checked": n, "max_ulp_vs_reference": worst}
    xs, w = host(wl.x[sel]), host(wl.w)
    # rows of whole 16-byte vectors run on the vector kernels, held to the fixed-order model
    vectors = (xs.shape[-1] * xs.dtype.itemsize) % 16 == 0
    full = None
    if wl.op == "rmsnorm_residual":
        rs = host(wl.r[sel])
        y_dev, ro_dev = wl.fn()
        y, ro = host(y_dev[sel]), host(ro_dev[sel])
        yo, roo = C.rmsnorm_residual(xs, rs, w, 1e-5, dt)
        ok = bool(np.array_equal(ro, roo))
        if vectors:
            # every row of the shard against the fixed-order model, bit for bit
            ym, rom = C.rmsnorm_fixed_order(host(wl.x), host(wl.r), w, 1e-5, dt, threads=threads)
            full = bool(np.array_equal(host(y_dev), ym) and np.array_equal(host(ro_dev), rom))
            ok = ok and full
        del y_dev, ro_dev
    else:
        y_dev = wl.fn()
        y = host(y_dev[sel])
        yo = C.rmsnorm(xs, w, 1e-6, dt)
        if vectors:
            full = bool(np.array_equal(host(y_dev), C.rmsnorm_fixed_order(host(wl.x), None, w, 1e-6, dt,
                                                                          threads=threads)))
            ok = full
        del y_dev
    worst = int(O.ulp_distance(yo, y, dt).max())
    ok = ok and worst <= (2 if dt != O.F32 else 6)
    return {"ok": ok, "rows": [wl.lo + i for i in sel], "max_ulp_vs_reference_order": worst,
            "all_rows_bit_exact_vs_fixed_order_model": full, "rows_checked_bit_exact": n if full is not None else 0}


# ------------------------------------------------------------- CPU baseline
def cpu_description() -> dict:
    model = platform.processor() or ""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_model": model, "os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads()}


def host_rows_that_fit(rows: int, hidden: int, element_size: int) -> int:
    """Rows of the workload AKO's CPU reference can run on in host memory: its
    inputs, outputs and fp32 temporaries (about 5 fp32 copies of a row) with a
    2x margin, within half of the memory available now."""
    try:
        avail = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
    except (ValueError, OSError):
        avail = 16 << 30
    per_row = hidden * (4 * element_size + 5 * 4) * 2
    fit = max(ROW_BLOCK, (avail // 2 // per_row) // ROW_BLOCK * ROW_BLOCK)
    return min(rows, fit)


def ako_reference_cpu(rows: int, hidden: int, dtype: torch.dtype, warmup: int, repeats: int) -> dict:
    """AKO's ``rmsnorm_residual_ref`` on CPU tensors of ``rows`` rows drawn
    like the workload's (N(0, 1) rows, N(1, 0.1) weight, from the CPU
    generator: the same distribution, not the GPU arm's bytes, which a
    memory-bound op's time does not depend on), timed with AKO's
    ``bench_op`` (wall clock on CPU, one call per timed batch, p50)."""
    from ako_b200.reference import ako

    ako()
    from ako.benchmark.bench_op import bench_op
    from ako.ops.rmsnorm_ref import rmsnorm_residual_ref

    # All the host threads this process may run on (a launcher such as
    # torchrun sets OMP_NUM_THREADS=1 for its ranks).
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    x, r = global_rows(0, rows, hidden, dtype, "cpu", 0)
    w = weight(hidden, dtype, "cpu", 0)
    res = bench_op(rmsnorm_residual_ref, (x, r, w), call_kwargs={"eps": 1e-5}, warmup=warmup, repeats=repeats,
                   inner=1, kernel_name="rmsnorm_residual_ref")
    b = x.element_size()
    nbytes = 4 * rows * hidden * b + hidden * b
    return {"value": round(nbytes / (res.latency_p50_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "cores": torch.get_num_threads(), "kind": "reference",
            "sample": f"{rows} x {hidden} {str(dtype).replace('torch.', '')} rows per call; AKO's "
                      f"ako.ops.rmsnorm_ref.rmsnorm_residual_ref on CPU tensors, timed by ako.benchmark.bench_op "
                      f"(warmup {warmup}, {repeats} timed calls, p50 {res.latency_p50_ms:.1f} ms)",
            "ms_per_call": round(res.latency_p50_ms, 3), "bytes_per_call": nbytes, **cpu_description()}


def c_port_cpu(rows: int, hidden: int, dtype: torch.dtype, seconds: float) -> dict:
    """The C restatement of AKO's reference (``oracle/ako_oracle.c``, all host
    threads) on ``rows`` rows drawn like the workload's."""
    import numpy as np

    from oracle import c_oracle as C

    x, r = global_rows(0, rows, hidden, dtype, "cpu", 0)
    w = weight(hidden, dtype, "cpu", 0)
    host = lambda t: t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()  # noqa: E731
    xn, rn, wn = host(x), host(r), host(w)
    name = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}[dtype]
    threads = C.default_threads()
    C.rmsnorm_residual(xn, rn, wn, 1e-5, name, threads=threads)  # page in, start threads
    calls, t0 = 0, time.perf_counter()
    while True:
        C.rmsnorm_residual(xn, rn, wn, 1e-5, name, threads=threads)
        calls += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    b = x.element_size()
    return {"value": round((4 * rows * hidden + hidden) * b * calls / dt / 1e9, 3), "unit": "GB/s",
            "cores": threads, "kind": "port",
            "sample": f"{rows} x {hidden} rows per call, {calls} calls in {dt:.1f} s "
                      f"(C restatement of AKO's reference, oracle/ako_oracle.c, pthreads)"}


# ---------------------------------------------------------------- extras
def run_ops(device: torch.device, peak: float) -> dict:
    from ako_b200.benchmark.timing import Flusher, cold_us

    flush = Flusher(device)
    out = {}
    for name in OPS_EXTRA:
        wl = Workload(name, device, seed=1)
        us = cold_us(wl.step, flush, n=10, blocks=3)
        gbs = wl.bytes / (us * 1e-6) / 1e9
        out[name] = {"op": wl.op, **wl.desc, "dtype": str(wl.dtype).replace("torch.", ""),
                     "bytes": wl.bytes, "us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                     "timing": "cold L2, differential (10 x (2xL2 read, call) - 10 x read) / 10"}
        del wl
        torch.cuda.empty_cache()
    return out


def run_decoder(reps: int) -> dict:
    """Configuration 5 on this GPU: the B200 decoder and the same stack on the
    reference math (``ako_b200.benchmark.decoder_bench``)."""
    from ako_b200.benchmark import decoder_bench

    args = argparse.Namespace(layers=4, prefill_batch=8, prefill_len=2048, decode_batch=32, decode_steps=128,
                              context=2048, warmup=2, reps=reps)
    res = decoder_bench.run(args)
    out = {"prefill_tok_s": res["b200"]["prefill_tok_s"], "decode_tok_s": res["b200"]["decode_tok_s"],
           "decode_graph_tok_s": res["b200"]["decode_graph_tok_s"], "b200": res["b200"],
           "reference_math": res["torch"], "parity": res["parity"],
           "speedup_vs_reference_math": res["speedup_vs_reference_math"],
           "config": "4 layers, d 4096, 32/8 heads, FFN 11008, bf16, N(0, 0.02) weights; prefill 8 x 2048; "
                     "decode 32 x 128 steps from a 2048-token cache; GEMMs and attention are torch's"}
    torch.cuda.empty_cache()
    return out


def run_ako_decoder() -> dict:
    """AKO's own decoder stack through AKO's selector, each mode in a fresh
    process with an empty kernel cache (``ako_b200.benchmark.ako_decoder``)."""
    import subprocess
    import tempfile

    with tempfile.TemporaryDirectory() as tmp:
        out = Path(tmp) / "ako_decoder.json"
        proc = subprocess.run([sys.executable, "-m", "ako_b200.benchmark.ako_decoder", "--reps", "3",
                               "--out", str(out)], cwd=str(REPO), capture_output=True, text=True, check=False)
        if proc.returncode != 0:
            return {"error": f"status {proc.returncode}: {proc.stderr.strip().splitlines()[-1:]}"}
        doc = json.loads(out.read_text())
    summary = {}
    for r in doc["results"]:
        chosen = [s["kernel"] for s in r.get("selections", [])]
        summary[r["mode"]] = {"prefill_tok_s": r["prefill_tok_s"], "decode_tok_s": r["decode_tok_s"],
                              "prefill_ms": r["prefill_ms"], "decode_ms_per_step": r["decode_ms_per_step"],
                              "selected": {k: chosen.count(k) for k in sorted(set(chosen))}}
    return summary


# ---------------------------------------------------------------- reference
def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the CPU reference runs once, on rank 0
    op, (m, h), dt = WORKLOADS[args.workload]
    if op != "rmsnorm_residual":
        raise SystemExit("--impl reference supports the rmsnorm_residual workloads")
    rows = host_rows_that_fit(m, h, torch.tensor([], dtype=dt).element_size())
    if args.reference_rows:
        rows = min(rows, args.reference_rows)
    ref = ako_reference_cpu(rows, h, dt, args.warmup, args.steps)
    port = c_port_cpu(rows, h, dt, min(10.0, args.cpu_seconds)) if not args.no_cpu else None
    value = ref["value"]
    line = {
        "impl": "reference", "metric": "achieved HBM GB/s", "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ref["ms_per_call"], "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) rows, weight N(1,0.1))",
        "config": {"workload": args.workload, "op": op, "rows": m, "hidden": h,
                   "step": f"one call of AKO's rmsnorm_residual_ref on CPU tensors of {rows} x {h} rows "
                           f"({'the whole batch' if rows == m else 'the rows host memory holds'}), drawn like the "
                           f"GPU arm's (seeded N(0,1) rows, N(1,0.1) weight, CPU generator)"},
        "cpu_baseline": {k: v for k, v in ref.items() if k not in ("ms_per_call", "bytes_per_call")},
        "c_port": port,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- main
def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--scaling", choices=("strong", "weak"), default="strong",
                    help="strong: one global batch split over the ranks; weak: a whole batch per rank")
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the host-buffer leg (default: --steps, max 20)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--reference-rows", type=int, default=None,
                    help="cap on the rows AKO's CPU reference runs on (default: as many as host memory holds)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ops", action="store_true")
    ap.add_argument("--no-decoder", action="store_true")
    ap.add_argument("--no-ako-decoder", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    if args.impl == "reference":
        run_reference(args)
        return

    from ako_b200 import _native, sharding
    from ako_b200.benchmark.clocks import start_sampler

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    peak, peak_src = hbm_peak()
    op, dims, _ = WORKLOADS[args.workload]
    row_op = op in ("rmsnorm", "rmsnorm_residual")
    strong = args.scaling == "strong"
    shard = sharding.shard_range(dims[0], world, rank) if strong else None

    wl = Workload(args.workload, device, seed=0, rows=shard)
    sampler = start_sampler(local)
    ms = timed_region(wl.step, args.steps, args.warmup, marks=sampler)
    clocks = sampler.stop()
    ms_max = sharding.max_over_ranks(ms, device)
    per_step_ms = ms_max / args.steps
    step_bytes = sharding.sum_over_ranks(wl.bytes, device)  # the global batch (strong) or N batches (weak)
    value = step_bytes / (per_step_ms * 1e-3) / 1e9
    achieved = wl.bytes / ((ms / args.steps) * 1e-3) / 1e9  # this rank's kernel
    parity = shard_parity(wl, threads=max(1, len(os.sched_getaffinity(0)) // world))
    parity_all = sharding.all_over_ranks(parity["ok"], device)

    weak = None
    if world > 1 and strong:
        full = Workload(args.workload, device, seed=100 + rank)
        wms = timed_region(full.step, args.steps, args.warmup)
        wmax = sharding.max_over_ranks(wms, device)
        weak = {"value": round(full.bytes * world / (wmax / args.steps * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(wmax / args.steps, 4),
                "config": f"a whole batch on every rank ({world} batches per step)"}
        del full
        torch.cuda.empty_cache()

    e2e = None
    if not args.no_e2e and wl.op == "rmsnorm_residual":
        from ako_b200 import host

        k = args.e2e_steps or min(args.steps, 20)
        xh = torch.empty(wl.x.shape, dtype=wl.dtype, pin_memory=True)
        rh = torch.empty(wl.x.shape, dtype=wl.dtype, pin_memory=True)
        yh = torch.empty(wl.x.shape, dtype=wl.dtype, pin_memory=True)
        roh = torch.empty(wl.x.shape, dtype=wl.dtype, pin_memory=True)
        xh.copy_(wl.x)
        rh.copy_(wl.r)
        e2e_step = lambda: host.rmsnorm_residual_host(xh, rh, wl.w, 1e-5, y_out=yh, residual_out=roh)  # noqa: E731
        ems = timed_region(e2e_step, k, 3)
        ems_max = sharding.max_over_ranks(ems, device)
        n, h = wl.x.shape
        io = 2 * n * h * wl.element_size
        e2e = {"value": round(step_bytes / (ems_max / k * 1e-3) / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": io * world, "d2h_bytes_per_step": io * world, "steps": k,
               "ms_per_step": round(ems_max / k, 3),
               "api": "ako_b200.host.rmsnorm_residual_host (pinned host buffers, chunked H2D/kernel/D2H "
                      "on three streams, C-ABI ako_b200_rmsnorm_residual per chunk)",
               "gpu_launches": k * world * host.launches_per_call(n, h, wl.element_size)}
        # The host path splits the rows into chunks; RMSNorm's summation order
        # does not depend on the row count, so its outputs must equal the
        # device call's bit for bit.
        y_dev, ro_dev = wl.fn()
        same = bool(torch.equal(yh, y_dev.cpu()) and torch.equal(roh, ro_dev.cpu()))
        e2e["outputs_equal_device_call"] = sharding.all_over_ranks(same, device)
        del xh, rh, yh, roh, y_dev, ro_dev

    # Every rank has finished its GPU work with the same collective steps; the
    # legs below run on rank 0 alone at N = 1.
    device_status = _native.take_device_status()
    sharding.finish()
    if rank != 0:
        return

    # GPU legs first: the CPU legs leave torch's intra-op threads spinning,
    # which slows the host's launches of short kernels that follow.
    ops = run_ops(device, peak) if world == 1 and not args.no_ops else None
    decoder = None
    if world == 1 and not args.no_decoder:
        decoder = run_decoder(reps=5)
        if not args.no_ako_decoder:
            decoder["ako_stack_through_akos_selector"] = run_ako_decoder()

    cpu = None
    if world == 1 and not args.no_cpu and wl.op == "rmsnorm_residual":
        m, h = dims
        rows = min(host_rows_that_fit(m, h, wl.element_size), 8192)
        cpu = ako_reference_cpu(rows, h, wl.dtype, warmup=1, repeats=3)
        cpu.pop("bytes_per_call", None)
        cpu["port"] = c_port_cpu(min(rows, 2048), h, wl.dtype, args.cpu_seconds)

    traffic = ncu_traffic(args.workload)
    line = {
        "metric": "achieved HBM GB/s",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per_step_ms, 4),
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": "bf16" if wl.dtype == torch.bfloat16 else str(wl.dtype).replace("torch.", ""),
        "data": "synthetic (seeded N(0,1) rows, weight N(1,0.1); N(0,2) SwiGLU inputs; generated on device by global row or batch index)",
        "config": {
            "workload": args.workload,
            "op": wl.op,
            **({"global_rows": dims[0], "rows_per_gpu": wl.hi - wl.lo, "hidden": dims[1]} if row_op else
               {**wl.desc, ("global_batch" if op.startswith("rope") else "global_rows"): dims[0]}),
            "bytes_per_step": step_bytes,
            "l2": "inputs larger than L2 (the step moves far more than the 126 MB L2); no flush",
            "parallelism": (f"one {dims[0]}-{'entry' if op.startswith('rope') else 'row'} batch split into {world} "
                            f"contiguous blocks (ako_b200.sharding.shard_range), no collective on the data path"
                            if strong else
                            f"a whole batch per rank x{world}, no collective on the data path"),
        },
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": traffic if world == 1 or not strong else None,
            "peak_source": peak_src,
            "frac_of_nominal_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
            "kernel": f"{wl.kernel} (CUDA events over the timed steps, launching stream, rank 0)",
        },
        "parity": ({**parity, "ok_all_ranks": parity_all} if parity is not None else None),
        "device_status": device_status,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "clocks": clocks,
        "gpu_launches": args.steps * world,
        "gpu_name": torch.cuda.get_device_name(device),
    }
    if weak is not None:
        line["weak"] = weak
    if ops is not None:
        line["ops"] = ops
    if decoder is not None:
        line["decoder"] = decoder
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
