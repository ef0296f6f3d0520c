"""Host-buffer entry points: row ops on tensors that live in (pinned) host memory.

The rows are streamed through the GPU in chunks on three CUDA streams —
host-to-device copies, the kernel, device-to-host copies — with a ring of
device slots, so the copies of one chunk overlap the kernel and the opposite
copies of its neighbours. PCIe (not HBM) bounds these calls; they exist so a
caller holding host data pays one call, and so the benchmark can time the
whole path a host caller sees.

The kernels are called through the C ABI (``ako_b200_rmsnorm_residual``)
on device slot buffers. A slot set is allocated once per (device, capacity,
hidden size, dtype, slot count), where the capacity in rows is the chunk
size, or for calls with fewer rows the next power of two at or above their
row count; at most ``MAX_SLOT_SETS`` sets are kept (least recently used
first out, after its streams have drained), so callers with varying batch
sizes do not accumulate device memory.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass

import torch

from ako_b200 import _native
from ako_b200.kernels import _DTYPE_CODE, MAX_HIDDEN_DIM

# Per operand per chunk. A call's first host-to-device chunk and last
# device-to-host chunk cannot overlap the other direction, so smaller chunks
# lose less at the ends but pay more per-chunk overhead; on B200 over PCIe
# (32768 x 16384 bf16, three slots) 32 MB measured 95.1 GB/s against 93.8 for
# 64 MB, 94.2 for 16 MB and 91.5 for 8 MB (a bidirectional copy of the same
# bytes: 99.3).
DEFAULT_CHUNK_BYTES = 32 << 20
#: Slot sets kept at once (each is 4 operands x slots x capacity rows).
MAX_SLOT_SETS = 4


@dataclass
class _Slots:
    x: list[torch.Tensor]
    r: list[torch.Tensor]
    y: list[torch.Tensor]
    ro: list[torch.Tensor]
    s_in: torch.cuda.Stream
    s_run: torch.cuda.Stream
    s_out: torch.cuda.Stream
    ev_in: list[torch.cuda.Event]
    ev_run: list[torch.cuda.Event]
    ev_out: list[torch.cuda.Event]


_slot_cache: OrderedDict[tuple, _Slots] = OrderedDict()


def slot_capacity(rows: int, chunk_rows: int) -> int:
    """Rows a slot holds for a call of ``rows`` rows in chunks of ``chunk_rows``:
    the chunk, or the next power of two at or above a smaller call's rows."""
    if rows >= chunk_rows:
        return chunk_rows
    cap = 1
    while cap < rows:
        cap *= 2
    return min(cap, chunk_rows)


def _slots(device: torch.device, capacity: int, hidden: int, dtype: torch.dtype, n: int) -> _Slots:
    key = (device, capacity, hidden, dtype, n)
    s = _slot_cache.get(key)
    if s is not None:
        _slot_cache.move_to_end(key)
        return s
    while len(_slot_cache) >= MAX_SLOT_SETS:
        _, old = _slot_cache.popitem(last=False)
        for st in (old.s_in, old.s_run, old.s_out):
            st.synchronize()  # nothing in flight still uses its buffers
    mk = lambda: [torch.empty(capacity, hidden, dtype=dtype, device=device) for _ in range(n)]  # noqa: E731
    ev = lambda: [torch.cuda.Event() for _ in range(n)]  # noqa: E731
    s = _Slots(mk(), mk(), mk(), mk(), torch.cuda.Stream(device), torch.cuda.Stream(device),
               torch.cuda.Stream(device), ev(), ev(), ev())
    _slot_cache[key] = s
    return s


def rmsnorm_residual_host(
    x: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    *,
    y_out: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
    device: torch.device | str | None = None,
    chunk_rows: int | None = None,
    slots: int = 3,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused residual add + RMSNorm of host tensors on a B200; results land in host memory.

    ``x`` and ``residual`` are ``(..., hidden)`` CPU tensors (pinned for the
    copies to run asynchronously); ``weight`` is a device tensor on the target
    GPU (it is reused across calls). Outputs are written to ``y_out`` /
    ``residual_out`` (pinned CPU tensors) when given. The call is ordered after
    prior work on the device's current stream and the current stream waits for
    its last copy, so CUDA events on the current stream bracket it and a
    ``synchronize`` of that stream makes the outputs readable.
    """
    fn = "rmsnorm_residual_host"
    if x.is_cuda or residual.is_cuda:
        raise ValueError(f"{fn} takes host tensors; use rmsnorm_residual_cuda_sm100 for device tensors")
    if x.shape != residual.shape or x.dtype != residual.dtype:
        raise ValueError(f"Shape mismatch: x {tuple(x.shape)} vs residual {tuple(residual.shape)}")
    code = _DTYPE_CODE.get(x.dtype)
    if code is None:
        raise ValueError(f"{fn} supports float32/float16/bfloat16, got {x.dtype}")
    for name, t in (("y_out", y_out), ("residual_out", residual_out)):
        if t is not None and (t.shape != x.shape or t.dtype != x.dtype or t.is_cuda):
            raise ValueError(f"{fn}: {name} must be a host tensor of x's shape {tuple(x.shape)} and dtype {x.dtype}")
    dev = torch.device(device) if device is not None else weight.device
    if dev.type != "cuda" or weight.device != dev:
        raise ValueError(f"{fn}: weight must live on the target CUDA device")
    hidden = x.shape[-1]
    weight = _host_weight(weight, hidden, fn)
    wcode = _DTYPE_CODE.get(weight.dtype)
    if wcode is None:
        raise ValueError(f"{fn}: unsupported weight dtype {weight.dtype}")
    x2 = x.reshape(-1, hidden)
    r2 = residual.reshape(-1, hidden)
    rows = x2.shape[0]
    y = y_out if y_out is not None else torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    ro = residual_out if residual_out is not None else torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    y2, ro2 = y.view(-1, hidden), ro.view(-1, hidden)
    if rows == 0:
        return y, ro
    if chunk_rows is None:
        chunk_rows = max(1, DEFAULT_CHUNK_BYTES // max(1, hidden * x.element_size()))
    capacity = slot_capacity(rows, chunk_rows)
    chunk_rows = min(chunk_rows, rows)
    st = _slots(dev, capacity, hidden, x.dtype, slots)
    lib = _native.active()
    w_ptr = weight.data_ptr()
    with torch.cuda.device(dev):
        caller = torch.cuda.current_stream(dev)
        for s in (st.s_in, st.s_run, st.s_out):
            s.wait_stream(caller)
        for i, lo in enumerate(range(0, rows, chunk_rows)):
            k = i % slots
            n = min(chunk_rows, rows - lo)
            if i >= slots:
                st.s_in.wait_event(st.ev_run[k])  # kernel of the chunk that last used slot k read it
            with torch.cuda.stream(st.s_in):
                st.x[k][:n].copy_(x2[lo:lo + n], non_blocking=True)
                st.r[k][:n].copy_(r2[lo:lo + n], non_blocking=True)
                st.ev_in[k].record(st.s_in)
            st.s_run.wait_event(st.ev_in[k])
            if i >= slots:
                st.s_run.wait_event(st.ev_out[k])  # its outputs were copied out
            status = lib.ako_b200_rmsnorm_residual(
                st.x[k].data_ptr(), hidden, st.r[k].data_ptr(), hidden, w_ptr, wcode,
                st.y[k].data_ptr(), hidden, st.ro[k].data_ptr(), hidden,
                n, hidden, float(eps), code, st.s_run.cuda_stream,
            )
            _native.raise_for_status(status, fn)
            st.ev_run[k].record(st.s_run)
            st.s_out.wait_event(st.ev_run[k])
            with torch.cuda.stream(st.s_out):
                y2[lo:lo + n].copy_(st.y[k][:n], non_blocking=True)
                ro2[lo:lo + n].copy_(st.ro[k][:n], non_blocking=True)
                st.ev_out[k].record(st.s_out)
        caller.wait_stream(st.s_out)
    return y, ro


def _host_weight(weight: torch.Tensor, hidden: int, fn: str) -> torch.Tensor:
    """The weight as the C ABI takes it: ``(hidden,)`` and contiguous (a strided
    view is copied, as the device wrappers do)."""
    if hidden > MAX_HIDDEN_DIM:
        raise ValueError(f"{fn} supports hidden_dim <= {MAX_HIDDEN_DIM}, got {hidden}")
    if weight.shape != (hidden,):
        raise ValueError(f"Expected weight of shape ({hidden},), got {tuple(weight.shape)}")
    return weight if weight.stride(0) == 1 else weight.contiguous()


def launches_per_call(rows: int, hidden: int, element_size: int, chunk_rows: int | None = None) -> int:
    """Kernel launches one host call makes (one per chunk)."""
    if chunk_rows is None:
        chunk_rows = max(1, DEFAULT_CHUNK_BYTES // max(1, hidden * element_size))
    return -(-rows // min(chunk_rows, rows)) if rows else 0
