"""Public op API with measured dispatch: ``rmsnorm``, ``rmsnorm_residual``,
``rope``, ``rope_qk``, ``swiglu`` and ``build_rope_tables``.

Same signatures and dispatch as the reference's ``ako.ops`` wrappers
(``ako/ops/rmsnorm.py:11-56``, ``rope.py:12-58``, ``swiglu.py:11-24``):
each call registers the candidates once, asks the process-wide selector for
the kernel of this (op, shape, dtype, device), and calls it positionally.
``kernel=`` forces a candidate by name, e.g. ``kernel="rmsnorm_cuda_sm100"``.
"""

from __future__ import annotations

import torch

from ako_b200 import _native
from ako_b200.dispatch import references as refs
from ako_b200.dispatch.registry import KernelEntry, KernelRegistry, get_registry
from ako_b200.dispatch.selector import get_selector
from ako_b200.dispatch.references import build_rope_tables

_PYTORCH_PRIORITY = 10
_BASELINE_PRIORITY = 7
_registered = False


def register_all(registry: KernelRegistry | None = None, *, force: bool = False) -> KernelRegistry:
    """References (priority 10), torch baselines (7) and the CUDA kernels (6)."""
    global _registered
    reg = registry if registry is not None else get_registry()
    if registry is None and _registered and not force:
        return reg
    entries = [
        ("rmsnorm", "rmsnorm_ref", refs.rmsnorm_ref, "pytorch", _PYTORCH_PRIORITY),
        ("rmsnorm_residual", "rmsnorm_residual_ref", refs.rmsnorm_residual_ref, "pytorch", _PYTORCH_PRIORITY),
        ("rope", "rope_ref", refs.rope_ref, "pytorch", _PYTORCH_PRIORITY),
        ("swiglu", "swiglu_ref", refs.swiglu_ref, "pytorch", _PYTORCH_PRIORITY),
        ("rope_qk", "rope_qk_ref", refs.rope_qk_ref, "pytorch", _PYTORCH_PRIORITY),
        ("rmsnorm", "rmsnorm_torch_native", refs.rmsnorm_torch_native, "torch_native", _BASELINE_PRIORITY),
    ]
    if refs.compile_enabled():
        entries += [
            ("rmsnorm", "rmsnorm_compiled", refs.rmsnorm_compiled, "torch_compile", _BASELINE_PRIORITY),
            ("rmsnorm_residual", "rmsnorm_residual_compiled", refs.rmsnorm_residual_compiled, "torch_compile",
             _BASELINE_PRIORITY),
            ("rope", "rope_compiled", refs.rope_compiled, "torch_compile", _BASELINE_PRIORITY),
            ("swiglu", "swiglu_compiled", refs.swiglu_compiled, "torch_compile", _BASELINE_PRIORITY),
            ("rope_qk", "rope_qk_compiled", refs.rope_qk_compiled, "torch_compile", _BASELINE_PRIORITY),
        ]
    for op, name, fn, backend, prio in entries:
        reg.register(KernelEntry(op, name, fn, backend, prio))
    if torch.cuda.is_available():
        _native.lib()  # a GPU machine without the built library fails here, loudly
    from ako_b200.plugin import register

    register(reg, target="mirror")
    if registry is None:
        _registered = True
        get_selector().clear_memo()
    return reg


def reset_registration() -> None:
    global _registered
    _registered = False


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, *, kernel: str | None = None) -> torch.Tensor:
    register_all()
    return get_selector().select("rmsnorm", x, weight, forced=kernel)(x, weight, eps)


def rmsnorm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, *,
                     kernel: str | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    register_all()
    return get_selector().select("rmsnorm_residual", x, residual, weight, forced=kernel)(x, residual, weight, eps)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, style: str = "neox", *,
         kernel: str | None = None) -> torch.Tensor:
    register_all()
    fn = get_selector().select("rope", x, cos, sin, forced=kernel, extra_key=style, call_kwargs={"style": style})
    return fn(x, cos, sin, style)


def rope_qk(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, style: str = "neox", *,
            kernel: str | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE of a query/key pair, dispatched as one op (``rope_qk``).

    The reference applies ``rope`` twice (``ako/ops/rope.py:45-58``); here the
    pair is one dispatched op whose CUDA candidate is a single launch. A
    ``kernel=`` naming a ``rope`` candidate keeps the reference's two calls.
    """
    register_all()
    if kernel is not None and get_registry().get("rope", kernel) is not None:
        return rope(q, cos, sin, style, kernel=kernel), rope(k, cos, sin, style, kernel=kernel)
    fn = get_selector().select("rope_qk", q, k, cos, sin, forced=kernel, extra_key=style,
                               call_kwargs={"style": style})
    return fn(q, k, cos, sin, style)


def swiglu(gate: torch.Tensor, up: torch.Tensor, *, kernel: str | None = None) -> torch.Tensor:
    register_all()
    return get_selector().select("swiglu", gate, up, forced=kernel)(gate, up)


__all__ = ["build_rope_tables", "register_all", "rmsnorm", "rmsnorm_residual", "rope", "rope_qk", "swiglu"]
