"""Registration of the sm_100a kernels as candidates in AKO's dispatcher.

:func:`register` is the drop-in. It adds one ``KernelEntry`` per op to AKO's
registry (``ako.dispatcher.registry.get_registry()``): backend ``"cuda"``,
priority 6 (below AKO's pytorch reference at 10, so the reference stays the
unmeasured default, above its Triton kernels at 5). It then clears the
process-wide selector memo, as the reference's extension guide prescribes
(``docs/EXTENDING.md`` §1-3). It also registers ``rope_qk`` as a dispatched op
of its own: AKO's ``rope_qk`` is two ``rope`` calls (``ako/ops/rope.py:45-58``),
and the fused kernel needs an op name to compete under.

Two opt-ins make AKO's selector sound on B200 without modifying AKO:

* ``b200_timing=True`` sizes the L2 flush of AKO's ``bench_op``
  (``ako/benchmark/bench_op.py:155``, 32 MiB for a 4 MiB consumer L2) to twice
  this device's L2 (2 x 126 MB on B200), so every candidate is timed from a
  cold L2 instead of from the warm cache most benchmark cells fit in;
* ``shared_cache=True`` gives AKO's selector a
  :class:`ako_b200.shared_cache.LockedKernelCache`: the same
  ``kernel_cache.json`` document, but saves take an exclusive file lock and
  merge with what other processes wrote, where AKO's own save
  (``ako/dispatcher/cache.py:110-116``) rewrites the whole file from one
  process's memory and drops the records of the others (one process per GPU
  sharing ``AKO_CACHE_PATH``).
"""

from __future__ import annotations

import importlib
from typing import Any

import torch

from ako_b200 import kernels
from ako_b200.reference import ako

CUDA_BACKEND = "cuda"
CUDA_PRIORITY = 6
#: Priority of the reference baselines in AKO's registry (``ako/ops/_registry.py:17``).
REFERENCE_PRIORITY = 10
#: The L2 flush is this many times the device's L2 with ``b200_timing``.
FLUSH_L2_MULTIPLE = 2


def rope_qk_ref(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                style: str = "neox") -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's ``rope_qk`` computation: AKO's ``rope_ref`` on q, then on k.
    The validation baseline of the dispatched ``rope_qk`` op."""
    ako()
    from ako.ops.rope_ref import rope_ref

    return rope_ref(q, cos, sin, style), rope_ref(k, cos, sin, style)


def register(registry: Any = None, *, priority: int = CUDA_PRIORITY, b200_timing: bool = False,
             shared_cache: bool = False) -> Any:
    """Register the CUDA candidates in AKO's registry; returns the registry used.

    ``registry``: a registry of AKO's type to fill instead of the global one
    (the global selector is then left alone). ``b200_timing`` and
    ``shared_cache``: see the module docstring.
    """
    ako()
    from ako.dispatcher.registry import KernelEntry, get_registry
    from ako.dispatcher.selector import get_selector

    reg = registry if registry is not None else get_registry()
    for op_name, kernel_name, fn in kernels.CANDIDATES:
        reg.register(KernelEntry(op_name=op_name, kernel_name=kernel_name, fn=fn, backend=CUDA_BACKEND,
                                 priority=priority))
    reg.register(KernelEntry(op_name="rope_qk", kernel_name="rope_qk_ref", fn=rope_qk_ref, backend="pytorch",
                             priority=REFERENCE_PRIORITY))
    if registry is None:
        selector = get_selector()
        if b200_timing:
            use_b200_l2_flush()
        if shared_cache:
            from ako_b200.shared_cache import LockedKernelCache

            if not isinstance(selector.cache, LockedKernelCache):
                selector.cache = LockedKernelCache(selector.cache.path)
        selector.clear_memo()
    return reg


def use_b200_l2_flush(device: torch.device | str | None = None) -> int:
    """Size AKO's ``bench_op`` L2 flush to ``FLUSH_L2_MULTIPLE`` x this device's
    L2 and drop its cached flush buffer and flush cost; returns the new size."""
    ako()
    # the module, not the function of the same name that ako.benchmark re-exports
    ako_bench = importlib.import_module("ako.benchmark.bench_op")
    from ako.dispatcher import hardware

    l2 = hardware.get_device_info(device).l2_bytes
    if not l2:
        raise RuntimeError("use_b200_l2_flush: the device reports no L2 size")
    size = FLUSH_L2_MULTIPLE * int(l2)
    if ako_bench.L2_FLUSH_BYTES != size:
        ako_bench.L2_FLUSH_BYTES = size
        ako_bench._flush_buffer.cache_clear()
        ako_bench._flush_cost_ms.cache_clear()
    return size
