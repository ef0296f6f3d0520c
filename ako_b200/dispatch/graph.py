"""CUDA-graph capture of one candidate call, for timing decode-sized rows.

Same contract as the reference's ``ako/benchmark/graph.py:31-67``: warm up on
a side stream, capture one call, and return a replay callable, or an
uncaptured result with the reason (CPU tensors, or a capture that raised).
The caller keeps ``args`` alive for as long as it replays.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

import torch


@dataclass
class CapturedKernel:
    replay: Callable[[], None] | None
    captured: bool
    reason: str | None = None
    graph: Any = None
    output: Any = None


def try_capture(fn: Callable[..., Any], args: tuple[Any, ...], kwargs: dict[str, Any] | None = None,
                *, warmup: int = 3) -> CapturedKernel:
    kwargs = kwargs or {}
    x = args[0] if args else None
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        return CapturedKernel(None, False, "not_cuda")
    try:
        side = torch.cuda.Stream(x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn(*args, **kwargs)
        torch.cuda.current_stream(x.device).wait_stream(side)
        torch.cuda.synchronize(x.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = fn(*args, **kwargs)
        torch.cuda.synchronize(x.device)
    except RuntimeError as exc:
        return CapturedKernel(None, False, f"{type(exc).__name__}: {exc}")
    return CapturedKernel(g.replay, True, None, g, out)
