"""AKO ``KernelFn`` wrappers around the sm_100a C ABI.

Each function has the exact positional signature AKO's dispatcher calls a
candidate with (reference ``docs/EXTENDING.md`` §2; call sites
``ako/ops/rmsnorm.py:31,56``, ``ako/ops/rope.py:42``, ``ako/ops/swiglu.py:24``):

==================  =====================================  ==========================
op                  call                                   returns
==================  =====================================  ==========================
rmsnorm             ``fn(x, weight, eps)``                 tensor like ``x``
rmsnorm_residual    ``fn(x, residual, weight, eps)``       ``(normed, x + residual)``
rope                ``fn(x, cos, sin, style)``             tensor like ``x``
swiglu              ``fn(gate, up)``                       tensor like ``gate``
==================  =====================================  ==========================

Inputs are read-only; outputs are new tensors from torch's caching allocator.
The kernel is launched on the current CUDA stream of the input's device and
nothing synchronizes, so every wrapper can be captured in a CUDA graph.

Errors follow the reference's Triton wrappers (``ako/ops/rmsnorm_triton.py:123-136``,
``ako/ops/rope_triton.py:114-133``): shape, dtype and device problems raise
``ValueError`` (a CPU tensor included: there is no CPU fallback), a failed launch
raises ``RuntimeError``. AKO's selector records either as a rejection.
"""

from __future__ import annotations

import torch

from ako_b200 import _native

#: Widest row the wrappers accept, kept equal to the reference's limit
#: (``ako/ops/rmsnorm_triton.py:28``) so both candidates reject the same keys.
MAX_HIDDEN_DIM = 65536

ROPE_STYLES = ("neox", "interleaved")

_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
_STYLE_CODE = {"neox": 0, "interleaved": 1}

_current_stream = torch._C._cuda_getCurrentRawStream if hasattr(torch._C, "_cuda_getCurrentRawStream") else None


def _stream(device: torch.device) -> int:
    index = device.index if device.index is not None else torch.cuda.current_device()
    if _current_stream is not None:
        return _current_stream(index)
    return torch.cuda.current_stream(device).cuda_stream


def _dtype_code(t: torch.Tensor, name: str, fn: str) -> int:
    code = _DTYPE_CODE.get(t.dtype)
    if code is None:
        raise ValueError(f"{fn} supports float32/float16/bfloat16 {name}, got {t.dtype}")
    return code


def _require_cuda(t: torch.Tensor, fn: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{fn} requires a CUDA tensor")


def _rows_view(t: torch.Tensor, hidden: int) -> torch.Tensor:
    """2-D ``(rows, hidden)`` view with unit inner stride, copying only if no view exists."""
    if t.stride(-1) != 1 and t.numel() > 0:
        t = t.contiguous()
    try:
        return t.view(-1, hidden)
    except RuntimeError:
        return t.contiguous().view(-1, hidden)


def _row_stride(t2: torch.Tensor) -> int:
    return t2.stride(0) if t2.shape[0] > 1 else t2.shape[1]


def _check_weight(weight: torch.Tensor, x: torch.Tensor, hidden: int, fn: str) -> torch.Tensor:
    if hidden > MAX_HIDDEN_DIM:
        raise ValueError(f"{fn} supports hidden_dim <= {MAX_HIDDEN_DIM}, got {hidden}")
    if weight.shape != (hidden,):
        raise ValueError(f"Expected weight of shape ({hidden},), got {tuple(weight.shape)}")
    if weight.device != x.device:
        raise ValueError(f"{fn}: weight is on {weight.device}, x on {x.device}")
    return weight if weight.stride(0) == 1 else weight.contiguous()


class _DeviceGuard:
    """Makes ``device`` current for the launch when it is not already."""

    __slots__ = ("index", "prev")

    def __init__(self, device: torch.device) -> None:
        self.index = device.index
        self.prev = None

    def __enter__(self) -> None:
        if self.index is not None:
            cur = torch.cuda.current_device()
            if cur != self.index:
                self.prev = cur
                torch.cuda.set_device(self.index)

    def __exit__(self, *exc: object) -> None:
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def rmsnorm_cuda_sm100(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm on B200: ``(x * rsqrt(mean(x^2) + eps)) * weight`` in fp32, one rounding.

    Same contract as ``rmsnorm_ref`` (``ako/ops/rmsnorm_ref.py:8-23``).
    """
    fn = "rmsnorm_cuda_sm100"
    _require_cuda(x, fn)
    code = _dtype_code(x, "x", fn)
    hidden = x.shape[-1] if x.dim() > 0 else 0
    weight = _check_weight(weight, x, hidden, fn)
    wcode = _dtype_code(weight, "weight", fn)
    x2 = _rows_view(x, hidden)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    y2 = y.view(-1, hidden)
    with _DeviceGuard(x.device):
        status = _native.active().ako_b200_rmsnorm(
            x2.data_ptr(), _row_stride(x2), weight.data_ptr(), wcode,
            y2.data_ptr(), _row_stride(y2), x2.shape[0], hidden, float(eps), code, _stream(x.device),
        )
    _native.raise_for_status(status, fn)
    return y


def rmsnorm_residual_cuda_sm100(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6
) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused residual add + RMSNorm on B200; returns ``(normed, x + residual)``.

    Same contract as ``rmsnorm_residual_ref`` (``ako/ops/rmsnorm_ref.py:26-50``):
    the new residual is rounded to the storage dtype before it is normalized.
    """
    fn = "rmsnorm_residual_cuda_sm100"
    _require_cuda(x, fn)
    if x.shape != residual.shape:
        raise ValueError(f"Shape mismatch: x {tuple(x.shape)} vs residual {tuple(residual.shape)}")
    if residual.dtype != x.dtype or residual.device != x.device:
        raise ValueError(f"{fn}: residual must match x in dtype and device")
    code = _dtype_code(x, "x", fn)
    hidden = x.shape[-1] if x.dim() > 0 else 0
    weight = _check_weight(weight, x, hidden, fn)
    wcode = _dtype_code(weight, "weight", fn)
    x2 = _rows_view(x, hidden)
    r2 = _rows_view(residual, hidden)
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    ro = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    y2 = y.view(-1, hidden)
    ro2 = ro.view(-1, hidden)
    with _DeviceGuard(x.device):
        status = _native.active().ako_b200_rmsnorm_residual(
            x2.data_ptr(), _row_stride(x2), r2.data_ptr(), _row_stride(r2), weight.data_ptr(), wcode,
            y2.data_ptr(), _row_stride(y2), ro2.data_ptr(), _row_stride(ro2),
            x2.shape[0], hidden, float(eps), code, _stream(x.device),
        )
    _native.raise_for_status(status, fn)
    return y, ro


def rope_cuda_sm100(
    x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, style: str = "neox"
) -> torch.Tensor:
    """RoPE on B200 for ``x`` of shape ``(batch, seq_len, n_heads, head_dim)``.

    Same contract and checks as ``rope_ref`` (``ako/ops/rope_ref.py:57-107``).
    Strided ``x`` (e.g. a ``(B, H, S, D)`` tensor passed as ``.transpose(1, 2)``)
    is read in place; the output keeps the input's memory layout when the
    input is dense, and is contiguous otherwise.
    """
    fn = "rope_cuda_sm100"
    if style not in ROPE_STYLES:
        raise ValueError(f"Unknown RoPE style '{style}', expected one of {ROPE_STYLES}")
    _require_cuda(x, fn)
    _check_rope_args(x, cos, sin, fn)
    code = _dtype_code(x, "x", fn)
    cos, sin = _rope_tables(cos, sin)
    x, y = _rope_out(x)
    batch, seq_len, n_heads, head_dim = x.shape
    with _DeviceGuard(x.device):
        status = _native.active().ako_b200_rope(
            x.data_ptr(), x.stride(0), x.stride(1), x.stride(2),
            cos.data_ptr(), sin.data_ptr(), cos.stride(0),
            y.data_ptr(), y.stride(0), y.stride(1), y.stride(2),
            batch, seq_len, n_heads, head_dim, _STYLE_CODE[style], code, _stream(x.device),
        )
    _native.raise_for_status(status, fn)
    return y


def _check_rope_args(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, fn: str) -> None:
    if x.ndim != 4:
        raise ValueError(f"Expected x of shape (batch, seq_len, n_heads, head_dim), got {tuple(x.shape)}")
    if x.shape[-1] % 2 != 0:
        raise ValueError(f"head_dim must be even, got {x.shape[-1]}")
    if cos.shape != sin.shape:
        raise ValueError(f"cos/sin shape mismatch: {tuple(cos.shape)} vs {tuple(sin.shape)}")
    if cos.shape != (x.shape[1], x.shape[-1] // 2):
        raise ValueError(f"Expected cos/sin of shape {(x.shape[1], x.shape[-1] // 2)}, got {tuple(cos.shape)}")
    if cos.device != x.device or sin.device != x.device:
        raise ValueError(f"{fn}: cos/sin must be on {x.device}")


def _rope_tables(cos: torch.Tensor, sin: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    if cos.dtype != torch.float32 or sin.dtype != torch.float32:
        cos, sin = cos.to(torch.float32), sin.to(torch.float32)
    if cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0):
        cos, sin = cos.contiguous(), sin.contiguous()
    return cos, sin


def _rope_out(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    if x.stride(-1) != 1:
        x = x.contiguous()
    y = torch.empty_like(x)
    if y.stride(-1) != 1:
        y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    return x, y


def rope_qk_cuda_sm100(
    q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, style: str = "neox"
) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE of a query/key pair in one launch; returns ``(rope(q), rope(k))``.

    Same result as two ``rope_cuda_sm100`` calls (and as the reference's
    ``rope_qk``, ``ako/ops/rope.py:45-58``), but each position's table values
    are read once for the q and k heads together.
    """
    fn = "rope_qk_cuda_sm100"
    if style not in ROPE_STYLES:
        raise ValueError(f"Unknown RoPE style '{style}', expected one of {ROPE_STYLES}")
    _require_cuda(q, fn)
    _check_rope_args(q, cos, sin, fn)
    _check_rope_args(k, cos, sin, fn)
    if k.shape[:2] != q.shape[:2] or k.shape[-1] != q.shape[-1] or k.dtype != q.dtype or k.device != q.device:
        raise ValueError(f"{fn}: q {tuple(q.shape)} and k {tuple(k.shape)} must share batch, seq_len, head_dim, dtype")
    code = _dtype_code(q, "q", fn)
    cos, sin = _rope_tables(cos, sin)
    q, qo = _rope_out(q)
    k, ko = _rope_out(k)
    batch, seq_len, qh, d = q.shape
    with _DeviceGuard(q.device):
        status = _native.active().ako_b200_rope_qk(
            q.data_ptr(), q.stride(0), q.stride(1), q.stride(2),
            k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
            cos.data_ptr(), sin.data_ptr(), cos.stride(0),
            qo.data_ptr(), qo.stride(0), qo.stride(1), qo.stride(2),
            ko.data_ptr(), ko.stride(0), ko.stride(1), ko.stride(2),
            batch, seq_len, qh, k.shape[2], d, _STYLE_CODE[style], code, _stream(q.device),
        )
    _native.raise_for_status(status, fn)
    return qo, ko


def swiglu_cuda_sm100(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """SwiGLU on B200: ``silu(gate) * up`` in fp32, one rounding.

    Same contract as ``swiglu_ref`` (``ako/ops/swiglu_ref.py:16-32``). Row-strided
    views (the two halves of a packed ``[M, 2F]`` projection) are read in place.
    """
    fn = "swiglu_cuda_sm100"
    _require_cuda(gate, fn)
    if gate.shape != up.shape:
        raise ValueError(f"Shape mismatch: gate {tuple(gate.shape)} vs up {tuple(up.shape)}")
    if up.dtype != gate.dtype or up.device != gate.device:
        raise ValueError(f"{fn}: up must match gate in dtype and device")
    code = _dtype_code(gate, "gate", fn)
    hidden = gate.shape[-1] if gate.dim() > 0 else 1
    if hidden > MAX_HIDDEN_DIM:
        raise ValueError(f"{fn} supports hidden_dim <= {MAX_HIDDEN_DIM}, got {hidden}")
    y = torch.empty(gate.shape, dtype=gate.dtype, device=gate.device)
    if gate.numel() == 0:
        return y
    g2 = _rows_view(gate.reshape(1) if gate.dim() == 0 else gate, hidden)
    u2 = _rows_view(up.reshape(1) if up.dim() == 0 else up, hidden)
    y2 = y.view(-1, hidden)
    with _DeviceGuard(gate.device):
        status = _native.active().ako_b200_swiglu(
            g2.data_ptr(), _row_stride(g2), u2.data_ptr(), _row_stride(u2),
            y2.data_ptr(), _row_stride(y2), g2.shape[0], hidden, code, _stream(gate.device),
        )
    _native.raise_for_status(status, fn)
    return y


#: (op_name, kernel_name, fn) for every candidate this package provides.
CANDIDATES = (
    ("rmsnorm", "rmsnorm_cuda_sm100", rmsnorm_cuda_sm100),
    ("rmsnorm_residual", "rmsnorm_residual_cuda_sm100", rmsnorm_residual_cuda_sm100),
    ("rope", "rope_cuda_sm100", rope_cuda_sm100),
    ("swiglu", "swiglu_cuda_sm100", swiglu_cuda_sm100),
    ("rope_qk", "rope_qk_cuda_sm100", rope_qk_cuda_sm100),
)
