"""Measured kernel selection: validate -> benchmark -> cache.

The selection rule and record of the reference's ``ako/dispatcher/selector.py``
(Algorithm 1 of the AKO paper), re-implemented:

1. a forced kernel name wins outright (unknown name: ``ValueError``);
2. a cached decision for ``(device key, op, shape key)`` is reused;
3. without autotuning (``AKO_AUTOTUNE=0``), on a non-CUDA device (unless
   ``allow_cpu_tuning``), or with a single candidate, the highest-priority
   entry is used;
4. otherwise the baseline (first ``backend == "pytorch"`` entry) is run and
   timed, every other candidate is run, rejected if its max error exceeds the
   dtype budget (or raises anything at all), else timed; the fastest survivor
   that beats the baseline by ``min_speedup`` is kept and written to the cache
   with the metrics that justified it.

``select`` memoizes the resolved function on cheap hashables (op, forced,
variant tag, dtype, shapes, device), so a repeated call costs a dict lookup.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any

import torch

from ako_b200.dispatch.bench_op import bench_op
from ako_b200.dispatch.cache import KernelCache
from ako_b200.dispatch.hardware import get_device_info
from ako_b200.dispatch.numerical import error_budget, error_in_ulps, max_abs_error_any
from ako_b200.dispatch.registry import KernelEntry, KernelFn, KernelRegistry, get_registry

#: Backends anyone could run without AKO; the quotable speedup is over the fastest of them.
BASELINE_BACKENDS = frozenset({"pytorch", "torch_native", "torch_compile"})


def _env_on(name: str, default: bool) -> bool:
    v = os.environ.get(name)
    return default if v is None else v.strip().lower() in {"1", "true", "yes", "on"}


def shape_key(tensors: tuple[torch.Tensor, ...], extra: str | None = None) -> str:
    """``"(shape)_dtype_(shape of each other arg)[_extra]"`` — the cache key of a call."""
    if not tensors:
        raise ValueError("At least one tensor is required to build a shape key")
    first = tensors[0]
    parts = [str(tuple(first.shape)), str(first.dtype).removeprefix("torch.")]
    parts += [str(tuple(t.shape)) for t in tensors[1:]]
    if extra:
        parts.append(extra)
    return "_".join(parts)


@dataclass(frozen=True)
class SelectionResult:
    op_name: str
    entry: KernelEntry
    shape_key: str
    source: str  # "forced" | "cache" | "default" | "benchmark"
    latency_p50_ms: float | None = None
    baseline_ms: float | None = None
    max_error: float | None = None
    candidates_evaluated: int = 0
    rejected: tuple[str, ...] = ()
    best_baseline_ms: float | None = None
    best_baseline_kernel: str | None = None

    @property
    def from_cache(self) -> bool:
        return self.source == "cache"

    @property
    def speedup(self) -> float | None:
        if self.baseline_ms and self.latency_p50_ms:
            return self.baseline_ms / self.latency_p50_ms
        return None

    @property
    def speedup_vs_best_baseline(self) -> float | None:
        if self.best_baseline_ms and self.latency_p50_ms:
            return self.best_baseline_ms / self.latency_p50_ms
        return None

    def to_dict(self) -> dict[str, Any]:
        sp, spb = self.speedup, self.speedup_vs_best_baseline
        return {
            "operation": self.op_name,
            "selected_kernel": self.entry.kernel_name,
            "backend": self.entry.backend,
            "shape_key": self.shape_key,
            "source": self.source,
            "from_cache": self.from_cache,
            "latency_p50_ms": self.latency_p50_ms,
            "baseline_ms": self.baseline_ms,
            "speedup": round(sp, 3) if sp else None,
            "best_baseline_ms": self.best_baseline_ms,
            "best_baseline_kernel": self.best_baseline_kernel,
            "speedup_vs_best_baseline": round(spb, 3) if spb else None,
            "max_error": self.max_error,
            "candidates_evaluated": self.candidates_evaluated,
            "rejected": list(self.rejected),
        }


class KernelSelector:
    def __init__(
        self,
        registry: KernelRegistry | None = None,
        cache: KernelCache | None = None,
        *,
        auto_tune: bool | None = None,
        error_threshold: float | None = None,
        min_speedup: float = 1.0,
        warmup: int = 5,
        repeats: int = 20,
        allow_cpu_tuning: bool = False,
    ) -> None:
        self.registry = registry if registry is not None else get_registry()
        self.cache = cache if cache is not None else KernelCache()
        self.auto_tune = _env_on("AKO_AUTOTUNE", True) if auto_tune is None else auto_tune
        self.error_threshold = error_threshold
        self.min_speedup = min_speedup
        self.warmup = warmup
        self.repeats = repeats
        self.allow_cpu_tuning = allow_cpu_tuning
        self._memo: dict[tuple[Any, ...], KernelFn] = {}

    def select(self, op_name: str, x: torch.Tensor, *args: torch.Tensor, forced: str | None = None,
               extra_key: str | None = None, call_kwargs: dict[str, Any] | None = None) -> KernelFn:
        key = (op_name, forced, extra_key, x.dtype, x.shape, x.device.type, x.device.index,
               tuple(a.shape for a in args))
        fn = self._memo.get(key)
        if fn is None:
            fn = self.select_entry(op_name, x, *args, forced=forced, extra_key=extra_key,
                                   call_kwargs=call_kwargs).entry.fn
            self._memo[key] = fn
        return fn

    def clear_memo(self) -> None:
        self._memo.clear()

    def select_entry(self, op_name: str, x: torch.Tensor, *args: torch.Tensor, forced: str | None = None,
                     extra_key: str | None = None, call_kwargs: dict[str, Any] | None = None) -> SelectionResult:
        candidates = self.registry.list_kernels(op_name)
        if not candidates:
            raise ValueError(f"No kernels registered for op '{op_name}'")
        key = shape_key((x, *args), extra_key)
        if forced:
            entry = self.registry.get(op_name, forced)
            if entry is None:
                names = ", ".join(c.kernel_name for c in candidates)
                raise ValueError(f"Unknown kernel '{forced}' for op '{op_name}' (available: {names})")
            return SelectionResult(op_name, entry, key, source="forced")

        gpu_key = get_device_info(x.device).cache_key
        rec = self.cache.get_record(gpu_key, op_name, key)
        if rec is not None:
            entry = self.registry.get(op_name, rec.get("kernel", ""))
            if entry is not None:
                return SelectionResult(
                    op_name, entry, key, source="cache", latency_p50_ms=rec.get("latency_p50_ms"),
                    baseline_ms=rec.get("baseline_ms"), max_error=rec.get("max_error"),
                    best_baseline_ms=rec.get("best_baseline_ms"), best_baseline_kernel=rec.get("best_baseline_kernel"),
                )

        tunable = x.device.type == "cuda" or self.allow_cpu_tuning
        if not self.auto_tune or not tunable or len(candidates) == 1:
            return SelectionResult(op_name, candidates[0], key, source="default")
        return self._measure(op_name, candidates, (x, *args), key, call_kwargs or {}, gpu_key)

    def _measure(self, op_name: str, candidates: list[KernelEntry], tensors: tuple[torch.Tensor, ...],
                 key: str, kwargs: dict[str, Any], gpu_key: str) -> SelectionResult:
        baseline = next((c for c in candidates if c.backend == "pytorch"), candidates[-1])
        reference = baseline.fn(*tensors, **kwargs)
        timing = lambda e: bench_op(e.fn, tensors, warmup=self.warmup, repeats=self.repeats,  # noqa: E731
                                    kernel_name=e.kernel_name, call_kwargs=kwargs).latency_p50_ms
        baseline_ms = timing(baseline)
        budget = error_budget(reference) if self.error_threshold is None else self.error_threshold

        best, best_ms, best_err = baseline, baseline_ms, 0.0
        evaluated = 1
        rejected: list[str] = []
        baselines = {baseline.kernel_name: baseline_ms}
        for cand in candidates:
            if cand.kernel_name == baseline.kernel_name:
                continue
            try:
                out = cand.fn(*tensors, **kwargs)
                err = max_abs_error_any(reference, out)
                if err > budget:
                    rejected.append(f"{cand.kernel_name}: max_error={err:.3e} > budget={budget:.3e} "
                                    f"({error_in_ulps(reference, out):.1f} ulps)")
                    continue
                ms = timing(cand)
            except Exception as exc:  # a broken candidate is a rejection, never a dispatch failure
                rejected.append(f"{cand.kernel_name}: {type(exc).__name__}: {exc}")
                continue
            evaluated += 1
            if cand.backend in BASELINE_BACKENDS:
                baselines[cand.kernel_name] = ms
            if ms < best_ms and baseline_ms >= ms * self.min_speedup:
                best, best_ms, best_err = cand, ms, err

        best_base = min(baselines, key=baselines.__getitem__)
        self.cache.set(
            gpu_key, op_name, key, best.kernel_name,
            latency_p50_ms=round(best_ms, 4),
            baseline_ms=round(baseline_ms, 4),
            speedup=round(baseline_ms / best_ms, 3) if best_ms > 0 else None,
            best_baseline_ms=round(baselines[best_base], 4),
            best_baseline_kernel=best_base,
            speedup_vs_best_baseline=round(baselines[best_base] / best_ms, 3) if best_ms > 0 else None,
            max_error=best_err,
            error_budget=budget,
            backend=best.backend,
        )
        return SelectionResult(op_name, best, key, source="benchmark", latency_p50_ms=best_ms,
                               baseline_ms=baseline_ms, max_error=best_err, candidates_evaluated=evaluated,
                               rejected=tuple(rejected), best_baseline_ms=baselines[best_base],
                               best_baseline_kernel=best_base)


_selector: KernelSelector | None = None


def get_selector() -> KernelSelector:
    global _selector
    if _selector is None:
        _selector = KernelSelector()
    return _selector


def reset_selector() -> None:
    global _selector
    _selector = None
