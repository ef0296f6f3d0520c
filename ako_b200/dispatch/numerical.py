"""Numerics gate of the selector: a dtype-scaled error budget and ulp reports.

Same definitions as the reference's ``ako/validation/numerical.py:20-122``:
``budget = tol_scale * (atol + rtol(dtype) * max|reference|)`` with the
``torch.testing`` default relative tolerances, and errors reported in units of
the output dtype's spacing at ``max|reference|``. :func:`ulp_distance` adds
the elementwise distance in representable steps.
"""

from __future__ import annotations

import math
from typing import Any, Sequence

import torch

DTYPE_RTOL: dict[torch.dtype, float] = {
    torch.float64: 1e-7,
    torch.float32: 1.3e-6,
    torch.float16: 1e-3,
    torch.bfloat16: 1.6e-2,
}
DEFAULT_ATOL = 1e-5


def max_abs_error(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a.float() - b.float()).abs().max().item() if a.numel() else 0.0


def max_abs_error_any(a: Any, b: Any) -> float:
    """Max abs error between two outputs: tensors or (nested) sequences of them."""
    if isinstance(a, torch.Tensor) and isinstance(b, torch.Tensor):
        return max_abs_error(a, b)
    if isinstance(a, Sequence) and isinstance(b, Sequence):
        if len(a) != len(b):
            raise ValueError(f"Output arity mismatch: {len(a)} vs {len(b)}")
        return max((max_abs_error_any(x, y) for x, y in zip(a, b)), default=0.0)
    raise TypeError(f"Cannot compare outputs of types {type(a)!r} and {type(b)!r}")


def _magnitude(ref: Any) -> tuple[float, torch.dtype]:
    if isinstance(ref, torch.Tensor):
        return (ref.float().abs().max().item() if ref.numel() else 0.0), ref.dtype
    if isinstance(ref, Sequence) and ref:
        parts = [_magnitude(r) for r in ref]
        return max(p[0] for p in parts), parts[0][1]
    raise TypeError(f"Cannot measure magnitude of {type(ref)!r}")


def ulp(dtype: torch.dtype, magnitude: float) -> float:
    """Spacing of representable ``dtype`` values in the binade of ``magnitude``."""
    info = torch.finfo(dtype)
    magnitude = abs(magnitude)
    if magnitude < info.tiny:
        return info.tiny
    return math.ldexp(info.eps, math.floor(math.log2(magnitude)))


def error_budget(reference: Any, *, rtol: float | None = None, atol: float = DEFAULT_ATOL,
                 tol_scale: float = 1.0) -> float:
    magnitude, dtype = _magnitude(reference)
    if rtol is None:
        rtol = DTYPE_RTOL.get(dtype, 1e-3)
    return tol_scale * (atol + rtol * magnitude)


def error_in_ulps(reference: Any, candidate: Any) -> float:
    magnitude, dtype = _magnitude(reference)
    return max_abs_error_any(reference, candidate) / ulp(dtype, magnitude)


def ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Elementwise |a - b| in representable steps of their (common) dtype."""
    if a.dtype != b.dtype:
        raise ValueError("ulp_distance needs tensors of one dtype")
    int_t = {torch.float32: torch.int32, torch.float16: torch.int16, torch.bfloat16: torch.int16,
             torch.float64: torch.int64}[a.dtype]
    sign = {torch.int32: 0x7FFFFFFF, torch.int16: 0x7FFF, torch.int64: 0x7FFFFFFFFFFFFFFF}[int_t]

    def ordered(t: torch.Tensor) -> torch.Tensor:
        i = t.contiguous().view(int_t).to(torch.int64)
        return torch.where(i < 0, -(i & sign), i)

    return (ordered(a) - ordered(b)).abs()
