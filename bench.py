#!/usr/bin/env python
"""Benchmark of the B200 kernels behind AKO's dispatcher API; prints ONE JSON line.

Metric: achieved HBM GB/s = algorithmic bytes / device time.
A step is one pass of the hot path over one batch: by default one fused
residual-add RMSNorm (``rmsnorm_residual``) over config 2's largest cell,
32768 rows x 16384 bf16 per GPU (4.3 GB moved per step, far above the 126 MB
L2, so back-to-back steps need no flush).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

* ``value``: whole-job GB/s, inputs resident in HBM, CUDA events on the
  launching stream around exactly K steps, max over ranks.
* ``e2e``: the same metric through the host-buffer call
  (``ako_b200.host.rmsnorm_residual_host``): pinned host inputs copied in and
  results copied out inside the timed region, every step.
* ``roofline``: the kernel's achieved bytes per launch / measured HBM copy
  bandwidth (``MEASURED_PEAKS.json``), with DRAM traffic from the committed
  ncu summary of this workload.
* ``cpu_baseline``: the C oracle (a restatement of AKO's unfused reference,
  all host threads) on a bounded row sample of the same workload, rank 0, N=1.
* ``ops``: the other ops at their largest benchmark cell (N=1), device time
  per call from a cold L2 (differential timing).

Multi-GPU (torchrun): every rank owns its own row shard (weak scaling); no
collective touches the data path, only the max of the timings.
``--impl reference`` times the CPU oracle port of AKO's reference (rank 0).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

BF16_BYTES = 2
FALLBACK_HBM_GBS = 6650.0
NOMINAL_HBM_GBS = 8000.0  # B200 HBM3e datasheet figure, the metric's "% of ~8 TB/s"
L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    # name: (op, dims, dtype)
    "rmsnorm_residual_bf16_32768x16384": ("rmsnorm_residual", (32768, 16384), torch.bfloat16),
    "rmsnorm_residual_bf16_32768x4096": ("rmsnorm_residual", (32768, 4096), torch.bfloat16),
    "rmsnorm_residual_bf16_8192x4096": ("rmsnorm_residual", (8192, 4096), torch.bfloat16),
    "rmsnorm_residual_bf16_4096x8192": ("rmsnorm_residual", (4096, 8192), torch.bfloat16),
    "rmsnorm_fp32_2048x4096": ("rmsnorm", (2048, 4096), torch.float32),
    "rope_q_bf16_32x4096x32x128": ("rope", (32, 4096, 32, 128), torch.bfloat16),
    "rope_k_bf16_32x4096x8x128": ("rope", (32, 4096, 8, 128), torch.bfloat16),
    "rope_q_bf16_8x512x32x128": ("rope", (8, 512, 32, 128), torch.bfloat16),
    "swiglu_bf16_16384x14336": ("swiglu", (16384, 14336), torch.bfloat16),
    "swiglu_packed_bf16_16384x14336": ("swiglu_packed", (16384, 14336), torch.bfloat16),
    "swiglu_bf16_2048x14336": ("swiglu", (2048, 14336), torch.bfloat16),
    "swiglu_packed_bf16_2048x14336": ("swiglu_packed", (2048, 14336), torch.bfloat16),
    # small cases of the same kernels (a few hundred MB, above L2) for ncu captures
    "rmsnorm_residual_bf16_2048x16384": ("rmsnorm_residual", (2048, 16384), torch.bfloat16),
    "rmsnorm_residual_bf16_4096x4096": ("rmsnorm_residual", (4096, 4096), torch.bfloat16),
    "rope_q_bf16_16x512x32x128": ("rope", (16, 512, 32, 128), torch.bfloat16),
}
DEFAULT_WORKLOAD = "rmsnorm_residual_bf16_32768x16384"
OPS_EXTRA = [
    "rmsnorm_fp32_2048x4096",
    "rmsnorm_residual_bf16_32768x4096",
    "rope_q_bf16_32x4096x32x128",
    "rope_k_bf16_32x4096x8x128",
    "swiglu_bf16_16384x14336",
    "swiglu_packed_bf16_16384x14336",
]


def log(*a: object) -> None:
    print(*a, file=sys.stderr, flush=True)


# ----------------------------------------------------------------- workloads
class Workload:
    """Inputs in HBM, one kernel launch per step, and its algorithmic bytes."""

    def __init__(self, name: str, device: torch.device, seed: int = 0) -> None:
        from ako_b200 import kernels

        self.name = name
        self.op, self.dims, self.dtype = WORKLOADS[name]
        b = torch.tensor([], dtype=self.dtype).element_size()
        g = torch.Generator(device=device).manual_seed(seed)
        rnd = lambda *s, mean=0.0, std=1.0: (torch.randn(*s, generator=g, device=device) * std + mean).to(self.dtype)  # noqa: E731
        if self.op in ("rmsnorm", "rmsnorm_residual"):
            m, h = self.dims
            self.x = rnd(m, h)
            self.w = rnd(h, mean=1.0, std=0.1)
            if self.op == "rmsnorm":
                self.bytes = 2 * m * h * b + h * b
                self.fn = lambda: kernels.rmsnorm_cuda_sm100(self.x, self.w, 1e-6)
            else:
                self.r = rnd(m, h)
                self.bytes = 4 * m * h * b + h * b
                self.fn = lambda: kernels.rmsnorm_residual_cuda_sm100(self.x, self.r, self.w, 1e-5)
            self.desc = {"rows": m, "hidden": h}
        elif self.op == "rope":
            bb, s, hh, d = self.dims
            from ako_b200.api import build_rope_tables

            cos, sin = build_rope_tables(8192, d, device=device)
            self.cos, self.sin = cos[:s], sin[:s]
            self.x = rnd(bb, s, hh, d)
            self.bytes = 2 * bb * s * hh * d * b + s * (d // 2) * 4 * 2
            self.fn = lambda: kernels.rope_cuda_sm100(self.x, self.cos, self.sin, "neox")
            self.desc = {"batch": bb, "seq": s, "heads": hh, "head_dim": d, "style": "neox", "table": "fp32 [8192, 64] sliced"}
        else:
            m, f = self.dims
            if self.op == "swiglu_packed":
                self.packed = rnd(m, 2 * f, std=2.0)
                self.g, self.u = self.packed[:, :f], self.packed[:, f:]
            else:
                self.g, self.u = rnd(m, f, std=2.0), rnd(m, f, std=2.0)
            self.bytes = 3 * m * f * b
            self.fn = lambda: kernels.swiglu_cuda_sm100(self.g, self.u)
            self.desc = {"rows": m, "hidden": f, "packed": self.op == "swiglu_packed"}
        self.launches_per_step = 1

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
            sharding.init("nccl", device=torch.device("cuda", local))
            sharding.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    return world, rank, local


def barrier(world: int) -> None:
    from ako_b200 import sharding

    sharding.barrier()


def max_over_ranks(v: float, world: int, device: torch.device) -> float:
    from ako_b200 import sharding

    return sharding.max_over_ranks(v, device)


def timed_region(step, k: int, w: int, world: int, marks=None) -> float:
    """W untimed steps, then exactly K steps between events; ms on this rank.
    ``marks`` (a clock sampler) gets the host times around the timed steps."""
    for _ in range(w):
        step()
    torch.cuda.synchronize()
    barrier(world)
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
    barrier(world)
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


def cpu_baseline(wl: Workload, seconds: float, sample_rows: int | None = None) -> dict:
    """C oracle (restated reference, all host threads) on a row sample of the workload."""
    from oracle import c_oracle as C

    m, h = wl.dims
    b = wl.x.element_size()
    rows = sample_rows or max(1, min(m, (256 << 20) // (4 * h * b)))
    to_np = lambda t: t.cpu().view(torch.int16).numpy().view("uint16") if t.dtype == torch.bfloat16 else t.cpu().numpy()  # noqa: E731
    x, r, w = to_np(wl.x[:rows]), to_np(wl.r[:rows]), to_np(wl.w)
    dtype = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}[wl.dtype]
    threads = C.default_threads()
    C.rmsnorm_residual(x, r, w, 1e-5, dtype, threads=threads)  # warm (page in, thread start)
    calls, t0 = 0, time.perf_counter()
    while True:
        C.rmsnorm_residual(x, r, w, 1e-5, dtype, threads=threads)
        calls += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    bytes_ = (4 * rows * h + h) * b * calls
    return {"value": round(bytes_ / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"rows 0..{rows - 1} of the {m}x{h} {dtype} workload, {calls} calls in {dt:.1f} s "
                      f"(C oracle, pthreads)"}


# ---------------------------------------------------------------- reference
def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the CPU reference runs once, on rank 0
    from oracle import c_oracle as C
    import numpy as np

    op, (m, h), dt = WORKLOADS[args.workload]
    if op != "rmsnorm_residual":
        raise SystemExit("--impl reference supports the rmsnorm_residual workloads")
    b = 2
    # ~256 MB of traffic per step, the cpu_baseline leg's sample: smaller
    # steps spend a larger share on starting the threads and touching fresh
    # output pages, which would understate the CPU's throughput.
    rows = max(1, min(m, (256 << 20) // (4 * h * b)))
    from oracle.ako_oracle import encode

    rng = np.random.default_rng(0)
    x = encode(rng.standard_normal((rows, h), dtype=np.float32), "bfloat16")
    r = encode(rng.standard_normal((rows, h), dtype=np.float32), "bfloat16")
    w = encode(rng.standard_normal(h, dtype=np.float32) * np.float32(0.1) + np.float32(1.0), "bfloat16")
    threads = C.default_threads()
    step = lambda: C.rmsnorm_residual(x, r, w, 1e-5, "bfloat16", threads=threads)  # noqa: E731
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    step_bytes = (4 * rows * h + h) * b
    value = step_bytes * args.steps / dt / 1e9
    line = {
        "impl": "reference", "metric": "achieved HBM GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1000 / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "op": op, "rows_per_gpu": m, "hidden": h,
                   "step": f"{rows}-row sample of the workload per step (bounded CPU work)"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{rows} x {h} bf16 rows per step; C restatement of AKO's unfused "
                                   f"reference (oracle/ako_oracle.c), pthreads"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
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
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the host-buffer leg (default: --steps, max 20)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ops", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    if args.impl == "reference":
        run_reference(args)
        return

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    peak, peak_src = hbm_peak()

    from ako_b200.benchmark.clocks import start_sampler

    wl = Workload(args.workload, device, seed=rank)
    sampler = start_sampler(local)
    ms = timed_region(wl.step, args.steps, args.warmup, world, marks=sampler)
    clocks = sampler.stop()
    ms_max = max_over_ranks(ms, world, device)
    per_step_ms = ms_max / args.steps
    total_bytes = wl.bytes * world
    value = total_bytes / (per_step_ms * 1e-3) / 1e9
    achieved = wl.bytes / ((ms / args.steps) * 1e-3) / 1e9  # this rank's kernel

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
        ems = timed_region(e2e_step, k, 3, world)
        ems_max = max_over_ranks(ems, world, device)
        m, h = wl.dims
        io = 2 * m * h * wl.x.element_size()
        e2e = {"value": round(total_bytes / (ems_max / k * 1e-3) / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": io, "d2h_bytes_per_step": io, "steps": k,
               "ms_per_step": round(ems_max / k, 3),
               "api": "ako_b200.host.rmsnorm_residual_host (pinned host buffers, chunked H2D/kernel/D2H "
                      "on three streams, C-ABI ako_b200_rmsnorm_residual per chunk)",
               "gpu_launches": k * host.launches_per_call(m, h, wl.x.element_size())}
        del xh, rh, yh, roh

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and wl.op == "rmsnorm_residual":
        cpu = cpu_baseline(wl, args.cpu_seconds)

    ops = None
    if world == 1 and not args.no_ops:
        ops = run_ops(device, peak)

    from ako_b200 import sharding

    sharding.finish()
    if rank != 0:
        return

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
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if wl.dtype == torch.bfloat16 else str(wl.dtype).replace("torch.", ""),
        "data": "synthetic (seeded N(0,1) inputs, weight N(1,0.1), generated on device)",
        "config": {
            "workload": args.workload,
            "op": wl.op,
            **{f"{k}_per_gpu" if k == "rows" else k: v for k, v in wl.desc.items()},
            "bytes_per_step_per_gpu": wl.bytes,
            "l2": "inputs larger than L2 (step moves far more than the 126 MB L2); no flush",
            "parallelism": f"row-sharded x{world}, no collective (weak scaling)",
        },
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": traffic,
            "peak_source": peak_src,
            "frac_of_nominal_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
            "kernel": "ako_b200::rms_rows_kernel (CUDA events over the timed steps, launching stream)",
        },
        "cpu_baseline": cpu,
        "e2e": e2e,
        "clocks": clocks,
        "gpu_launches": args.steps * wl.launches_per_step,
        "gpu_name": torch.cuda.get_device_name(device),
    }
    if ops is not None:
        line["ops"] = ops
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
