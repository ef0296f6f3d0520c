"""Validation baselines of the mirror selector (``backend == "pytorch"``).

These are the unfused definitions of the four ops in plain torch, the role the
reference's ``ako/ops/*_ref.py`` play in its registry: the selector runs the
first ``pytorch`` entry to get the numbers every candidate must match, and
uses it as the unmeasured default when autotuning is off. The CUDA candidates
(:mod:`ako_b200.kernels`) never call into this module.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F

ROPE_STYLES = ("neox", "interleaved")


def _compute_dtype(t: torch.Tensor) -> torch.dtype:
    return torch.float32 if t.dtype in (torch.float16, torch.bfloat16) else t.dtype


def rmsnorm_ref(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``(x * rsqrt(mean(x^2) + eps)) * weight`` in fp32 (fp64 stays fp64), cast back."""
    c = _compute_dtype(x)
    xc = x.to(c)
    inv = torch.rsqrt(xc.pow(2).mean(dim=-1, keepdim=True) + eps)
    return ((xc * inv) * weight.to(c)).to(x.dtype)


def rmsnorm_residual_ref(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                         eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
    """``new = x + residual`` (storage dtype), then ``(rmsnorm_ref(new), new)``."""
    if x.shape != residual.shape:
        raise ValueError(f"Shape mismatch: x {tuple(x.shape)} vs residual {tuple(residual.shape)}")
    new = x + residual
    return rmsnorm_ref(new, weight, eps), new


def build_rope_tables(seq_len: int, head_dim: int, *, base: float = 10000.0, offset: int = 0,
                      device: torch.device | str = "cpu", dtype: torch.dtype = torch.float32
                      ) -> tuple[torch.Tensor, torch.Tensor]:
    """``(cos, sin)`` of shape ``(seq_len, head_dim // 2)`` for positions ``offset..``.

    ``inv_freq = 1 / base ** (2i / head_dim)`` and ``angle = position * inv_freq``,
    both in fp32 (fp64 when ``dtype`` is fp64), then cast to ``dtype``.
    """
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even, got {head_dim}")
    c = torch.float64 if dtype == torch.float64 else torch.float32
    idx = torch.arange(0, head_dim // 2, device=device, dtype=c)
    inv_freq = 1.0 / (base ** (idx * 2.0 / head_dim))
    pos = torch.arange(offset, offset + seq_len, device=device, dtype=c)
    angles = torch.outer(pos, inv_freq)
    return angles.cos().to(dtype), angles.sin().to(dtype)


def _check_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, style: str) -> None:
    if style not in ROPE_STYLES:
        raise ValueError(f"Unknown RoPE style '{style}', expected one of {ROPE_STYLES}")
    if x.ndim != 4:
        raise ValueError(f"Expected x of shape (batch, seq_len, n_heads, head_dim), got {tuple(x.shape)}")
    d = x.shape[-1]
    if d % 2:
        raise ValueError(f"head_dim must be even, got {d}")
    if cos.shape != sin.shape:
        raise ValueError(f"cos/sin shape mismatch: {tuple(cos.shape)} vs {tuple(sin.shape)}")
    if cos.shape != (x.shape[1], d // 2):
        raise ValueError(f"Expected cos/sin of shape {(x.shape[1], d // 2)}, got {tuple(cos.shape)}")


def rope_ref(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, style: str = "neox") -> torch.Tensor:
    """Rotate pairs of ``x`` (batch, seq, heads, head_dim) by the table angles."""
    _check_rope(x, cos, sin, style)
    c = _compute_dtype(x)
    xc = x.to(c)
    cb = cos.to(c)[None, :, None, :]
    sb = sin.to(c)[None, :, None, :]
    if style == "neox":
        h = x.shape[-1] // 2
        a, b = xc[..., :h], xc[..., h:]
        out = torch.cat([a * cb - b * sb, a * sb + b * cb], dim=-1)
    else:
        a, b = xc[..., 0::2], xc[..., 1::2]
        out = torch.stack([a * cb - b * sb, a * sb + b * cb], dim=-1).flatten(-2)
    return out.to(x.dtype)


def rope_qk_ref(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                style: str = "neox") -> tuple[torch.Tensor, torch.Tensor]:
    """``(rope_ref(q), rope_ref(k))``: the reference's query/key pair, two calls."""
    return rope_ref(q, cos, sin, style), rope_ref(k, cos, sin, style)


def swiglu_ref(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` in fp32 (fp64 stays fp64), cast back."""
    if gate.shape != up.shape:
        raise ValueError(f"Shape mismatch: gate {tuple(gate.shape)} vs up {tuple(up.shape)}")
    c = _compute_dtype(gate)
    return (F.silu(gate.to(c)) * up.to(c)).to(gate.dtype)


def rmsnorm_torch_native(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """torch's fused ``F.rms_norm`` (a baseline, backend ``torch_native``)."""
    return F.rms_norm(x, (x.shape[-1],), weight, eps)


def compile_enabled() -> bool:
    return os.environ.get("AKO_ENABLE_COMPILE", "").strip().lower() in {"1", "true", "yes", "on"}


_compiled: dict[str, object] = {}


def _compiled_fn(name: str, fn):
    if name not in _compiled:
        _compiled[name] = torch.compile(fn, dynamic=True)
    return _compiled[name]


def rmsnorm_compiled(x, weight, eps=1e-6):
    return _compiled_fn("rmsnorm", rmsnorm_ref)(x, weight, eps)


def rmsnorm_residual_compiled(x, residual, weight, eps=1e-6):
    return _compiled_fn("rmsnorm_residual", rmsnorm_residual_ref)(x, residual, weight, eps)


def rope_compiled(x, cos, sin, style="neox"):
    return _compiled_fn("rope", rope_ref)(x, cos, sin, style)


def rope_qk_compiled(q, k, cos, sin, style="neox"):
    return _compiled_fn("rope_qk", rope_qk_ref)(q, k, cos, sin, style)


def swiglu_compiled(gate, up):
    return _compiled_fn("swiglu", swiglu_ref)(gate, up)
