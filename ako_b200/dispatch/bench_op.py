"""Timing primitive the selector uses to compare candidates.

Interface of the reference's ``ako/benchmark/bench_op.py:200-333``
(``bench_op(fn, args, *, warmup, repeats, kernel_name, call_kwargs, inner,
flush_l2, graph) -> BenchResult``): calls are timed in batches of about 1 ms
(at most 200 calls) so synchronization does not dominate; wall-clock latency
is what a caller pays, CUDA-event time is device time.

B200 difference: the L2 flush written before every call is twice the
device's L2 (2 x 126 MB on B200) instead of a fixed 32 MiB, so timings of
working sets that fit in 32 MiB-plus are not silently warm. The flush's own
cost is calibrated once per device and subtracted.
"""

from __future__ import annotations

import statistics
import time
from dataclasses import dataclass, field
from functools import lru_cache
from typing import Any, Callable

import torch

TARGET_BATCH_MS = 1.0
MAX_INNER_ITERS = 200
UNSTABLE_CV = 0.10
DEFAULT_L2_BYTES = 128 * 1024 * 1024


@dataclass(frozen=True)
class BenchResult:
    kernel_name: str
    shape: tuple[int, ...]
    dtype: str
    device: str
    latency_p50_ms: float
    latency_p95_ms: float
    latency_mean_ms: float
    latency_std_ms: float
    samples_ms: list[float] = field(repr=False)
    gpu_p50_ms: float | None = None
    inner_iters: int = 1
    peak_memory_mb: float | None = None
    l2_state: str = "n/a"
    l2_flush_ms: float = 0.0
    graph_captured: int = 0

    @property
    def launch_overhead_ms(self) -> float | None:
        return None if self.gpu_p50_ms is None else self.latency_p50_ms - self.gpu_p50_ms

    @property
    def cv(self) -> float:
        s = self.samples_ms
        m = statistics.mean(s) if s else 0.0
        return statistics.stdev(s) / m if len(s) > 1 and m > 0 else 0.0

    @property
    def unstable(self) -> bool:
        return self.cv > UNSTABLE_CV

    def to_dict(self) -> dict[str, Any]:
        d = {
            "kernel_name": self.kernel_name, "shape": list(self.shape), "dtype": self.dtype,
            "device": self.device, "latency_p50_ms": round(self.latency_p50_ms, 4),
            "latency_p95_ms": round(self.latency_p95_ms, 4), "latency_mean_ms": round(self.latency_mean_ms, 4),
            "latency_std_ms": round(self.latency_std_ms, 4), "inner_iters": self.inner_iters,
            "cv": round(self.cv, 4), "unstable": self.unstable, "l2_state": self.l2_state,
            "graph_captured": self.graph_captured, "samples_ms": [round(v, 7) for v in self.samples_ms],
        }
        if self.l2_flush_ms:
            d["l2_flush_ms"] = round(self.l2_flush_ms, 4)
        if self.gpu_p50_ms is not None:
            d["gpu_p50_ms"] = round(self.gpu_p50_ms, 4)
            d["launch_overhead_ms"] = round(self.latency_p50_ms - self.gpu_p50_ms, 4)
        if self.peak_memory_mb is not None:
            d["peak_memory_mb"] = round(self.peak_memory_mb, 2)
        return d


def _pct(values: list[float], p: float) -> float:
    if not values:
        return 0.0
    v = sorted(values)
    return v[min(int(len(v) * p), len(v) - 1)]


def l2_flush_bytes(device: torch.device) -> int:
    from ako_b200.dispatch.hardware import get_device_info

    l2 = get_device_info(device).l2_bytes or DEFAULT_L2_BYTES
    return 2 * int(l2)


@lru_cache(maxsize=None)
def _flush_buffer(device: torch.device) -> torch.Tensor:
    return torch.empty(l2_flush_bytes(device), dtype=torch.int8, device=device)


@lru_cache(maxsize=None)
def _flush_cost(device: torch.device) -> tuple[float, float]:
    """(wall ms, device ms) of one flush, measured once."""
    buf = _flush_buffer(device)
    r = bench_op(lambda b: b.zero_(), (buf,), warmup=3, repeats=10, inner=10, flush_l2=False,
                 kernel_name="l2_flush")
    return r.latency_p50_ms, r.gpu_p50_ms or 0.0


def _calibrate(fn: Callable[..., Any], args: tuple, kwargs: dict, cuda: bool) -> int:
    if cuda:
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    fn(*args, **kwargs)
    if cuda:
        torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1e3
    return MAX_INNER_ITERS if ms <= 0 else max(1, min(MAX_INNER_ITERS, int(TARGET_BATCH_MS / ms)))


def bench_op(
    fn: Callable[..., Any],
    args: tuple[Any, ...],
    *,
    warmup: int = 10,
    repeats: int = 50,
    kernel_name: str = "unknown",
    call_kwargs: dict[str, Any] | None = None,
    inner: int | None = None,
    flush_l2: bool = True,
    graph: bool = False,
) -> BenchResult:
    """Latency of one ``fn(*args, **call_kwargs)`` call, in ms (see module docstring)."""
    x = args[0]
    kwargs = call_kwargs or {}
    cuda = isinstance(x, torch.Tensor) and x.is_cuda
    flush = _flush_buffer(x.device) if (flush_l2 and cuda) else None
    flush_wall, flush_dev = _flush_cost(x.device) if flush is not None else (0.0, 0.0)

    for _ in range(warmup):
        fn(*args, **kwargs)
    if cuda:
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats(x.device)

    call = fn
    captured = 0
    if graph and cuda:
        from ako_b200.dispatch.graph import try_capture

        cap = try_capture(fn, args, kwargs)
        if cap.captured and cap.replay is not None:
            replay = cap.replay
            call = lambda *_a, **_k: replay()  # noqa: E731
            captured = 1
    if inner is None:
        inner = _calibrate(call, args, kwargs, cuda)

    samples: list[float] = []
    device_samples: list[float] = []
    for _ in range(repeats):
        if cuda:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            start.record()
            for _ in range(inner):
                if flush is not None:
                    flush.zero_()
                call(*args, **kwargs)
            end.record()
            torch.cuda.synchronize()
            wall = (time.perf_counter() - t0) * 1e3
            device_samples.append(max(start.elapsed_time(end) / inner - flush_dev, 0.0))
        else:
            t0 = time.perf_counter()
            for _ in range(inner):
                call(*args, **kwargs)
            wall = (time.perf_counter() - t0) * 1e3
        samples.append(max(wall / inner - flush_wall, 0.0))

    return BenchResult(
        kernel_name=kernel_name,
        shape=tuple(x.shape) if isinstance(x, torch.Tensor) else (),
        dtype=str(getattr(x, "dtype", "")).replace("torch.", ""),
        device=str(getattr(x, "device", "cpu")),
        latency_p50_ms=_pct(samples, 0.5),
        latency_p95_ms=_pct(samples, 0.95),
        latency_mean_ms=statistics.mean(samples),
        latency_std_ms=statistics.stdev(samples) if len(samples) > 1 else 0.0,
        samples_ms=samples,
        gpu_p50_ms=_pct(device_samples, 0.5) if device_samples else None,
        inner_iters=inner,
        peak_memory_mb=torch.cuda.max_memory_allocated(x.device) / 2**20 if cuda else None,
        l2_state="flushed" if flush is not None else ("off" if cuda else "n/a"),
        l2_flush_ms=flush_wall,
        graph_captured=captured,
    )
