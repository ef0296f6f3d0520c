"""Registration of the sm_100a kernels as candidates in AKO's dispatcher.

:func:`register` is the drop-in: with the reference package importable it
adds one ``KernelEntry`` per op to ``ako.dispatcher.registry.get_registry()``
(backend ``"cuda"``, priority 6: below AKO's pytorch reference at 10 so the
reference stays the unmeasured default, above its Triton kernels at 5) and
clears the process-wide selector memo, exactly as the reference's extension
guide prescribes (``docs/EXTENDING.md`` §1-3). Without it, the same entries go
into :mod:`ako_b200.dispatch`'s registry.
"""

from __future__ import annotations

from typing import Any

from ako_b200 import kernels

CUDA_BACKEND = "cuda"
CUDA_PRIORITY = 6


def ako_available() -> bool:
    try:
        import ako.dispatcher.registry  # noqa: F401
    except ImportError:
        return False
    return True


def register(registry: Any = None, *, priority: int = CUDA_PRIORITY, target: str = "auto") -> Any:
    """Register the CUDA candidates; returns the registry used.

    ``target``: ``"ako"`` (the reference's registry; ImportError if absent),
    ``"mirror"`` (:mod:`ako_b200.dispatch`), or ``"auto"`` (AKO when importable).
    An explicit ``registry`` receives entries of its own package's type.
    """
    use_ako = target == "ako" or (target == "auto" and registry is None and ako_available())
    if registry is not None:
        use_ako = type(registry).__module__.startswith("ako.")
    if use_ako:
        from ako.dispatcher.registry import KernelEntry, get_registry
        from ako.dispatcher.selector import get_selector
    else:
        from ako_b200.dispatch.registry import KernelEntry, get_registry
        from ako_b200.dispatch.selector import get_selector
    reg = registry if registry is not None else get_registry()
    for op_name, kernel_name, fn in kernels.CANDIDATES:
        reg.register(KernelEntry(op_name=op_name, kernel_name=kernel_name, fn=fn, backend=CUDA_BACKEND,
                                 priority=priority))
    if registry is None:
        get_selector().clear_memo()
    return reg
