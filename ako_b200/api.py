"""AKO's public op API with the sm_100a candidates registered.

``rmsnorm``, ``rmsnorm_residual``, ``rope`` and ``swiglu`` are AKO's own ops
(``ako/ops/rmsnorm.py:11-56``, ``rope.py:12-42``, ``swiglu.py:11-24``): the
first call registers AKO's kernels and then this package's candidates
(:func:`ako_b200.register`), and every call goes through AKO's process-wide
selector, cache and numerics gate. ``kernel=`` forces a candidate by name, e.g.
``kernel="rmsnorm_cuda_sm100"``.

``rope_qk`` is dispatched as an op of its own (``rope_qk``), whose reference
baseline is AKO's pair of ``rope_ref`` calls and whose CUDA candidate is one
launch for both tensors; ``kernel=`` naming a ``rope`` candidate keeps AKO's
two dispatched calls (``ako/ops/rope.py:45-58``).
"""

from __future__ import annotations

import threading

import torch

from ako_b200 import _native
from ako_b200.reference import ako

_lock = threading.Lock()
_ready = False


def _registered():
    """The reference package, with AKO's kernels and ours registered (once)."""
    global _ready
    pkg = ako()
    if _ready:
        return pkg
    with _lock:
        if not _ready:
            from ako.ops._registry import register_all

            from ako_b200.plugin import register

            register_all()
            register()
            if torch.cuda.is_available():
                _native.lib()  # a GPU machine without the built library fails here, loudly
            _ready = True
    return pkg


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, *, kernel: str | None = None) -> torch.Tensor:
    return _registered().rmsnorm(x, weight, eps, kernel=kernel)


def rmsnorm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, *,
                     kernel: str | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    return _registered().rmsnorm_residual(x, residual, weight, eps, kernel=kernel)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, style: str = "neox", *,
         kernel: str | None = None) -> torch.Tensor:
    return _registered().rope(x, cos, sin, style, kernel=kernel)


def rope_qk(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, style: str = "neox", *,
            kernel: str | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE of a query/key pair, dispatched as one op (``rope_qk``)."""
    pkg = _registered()
    from ako.dispatcher.registry import get_registry
    from ako.dispatcher.selector import get_selector

    if kernel is not None and get_registry().get("rope", kernel) is not None:
        return pkg.rope_qk(q, k, cos, sin, style, kernel=kernel)
    fn = get_selector().select("rope_qk", q, k, cos, sin, forced=kernel, extra_key=style,
                               call_kwargs={"style": style})
    return fn(q, k, cos, sin, style)


def swiglu(gate: torch.Tensor, up: torch.Tensor, *, kernel: str | None = None) -> torch.Tensor:
    return _registered().swiglu(gate, up, kernel=kernel)


def build_rope_tables(seq_len: int, head_dim: int, **kwargs) -> tuple[torch.Tensor, torch.Tensor]:
    """AKO's ``build_rope_tables`` (``ako/ops/rope_ref.py:20-54``): fp32 ``(cos, sin)``."""
    ako()
    from ako.ops.rope_ref import build_rope_tables as build

    return build(seq_len, head_dim, **kwargs)


__all__ = ["build_rope_tables", "rmsnorm", "rmsnorm_residual", "rope", "rope_qk", "swiglu"]
