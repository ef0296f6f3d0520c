"""Device timing of short launches with a cold L2.

CUDA event timestamps on the B200s measured here advance in steps of about
2 us, so a single launch bracketed by two events is quantized to that step,
and a launch whose outputs fit in L2 ends before they reach HBM.
:func:`cold_us` avoids both: it times ``n`` repetitions of (L2 flush, call)
between one pair of events, subtracts ``n`` flushes timed the same way, and
divides by ``n``. The flush is a read of twice the L2 size; it evicts the
previous call's outputs, so their write-back is charged to that call.
"""

from __future__ import annotations

import statistics
from typing import Callable

import torch

L2_FLUSH_BYTES = 2 * 126 * 1024 * 1024


class Flusher:
    """A 2 x L2 buffer on one device and a read of it (sum into a scalar)."""

    def __init__(self, device: torch.device, nbytes: int = L2_FLUSH_BYTES) -> None:
        self.buf = torch.empty(nbytes // 8, dtype=torch.int64, device=device)
        self.buf.zero_()
        self.sink = torch.empty((), dtype=torch.int64, device=device)

    def __call__(self) -> None:
        torch.sum(self.buf, dim=0, out=self.sink)


def _block_ms(body: Callable[[], None], n: int) -> float:
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(n):
        body()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e)


def cold_us(fn: Callable[[], object], flush: Flusher, n: int = 20, blocks: int = 5, warmup: int = 3) -> float:
    """Device time of one ``fn()`` starting from a cold L2, in microseconds."""
    for _ in range(warmup):
        fn()

    def both() -> None:
        flush()
        fn()

    samples = []
    for _ in range(blocks):
        t_both = _block_ms(both, n)
        t_flush = _block_ms(flush, n)
        samples.append((t_both - t_flush) * 1e3 / n)
    return max(statistics.median(samples), 0.0)


def back_to_back_us(fn: Callable[[], object], n: int = 50, blocks: int = 5, warmup: int = 3) -> float:
    """Device time per call of ``n`` calls issued back to back (warm L2 when inputs fit)."""
    for _ in range(warmup):
        fn()
    return statistics.median(_block_ms(fn, n) * 1e3 / n for _ in range(blocks))
