"""CPU oracle for the hot path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of AKO's unfused PyTorch references, used by ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` as the
checker. The product path (``ako_b200``) never imports this module.

Pinned: ``tests/test_oracle_golden.py`` checks it against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's own
functions (``ako.ops.*_ref``) on seeded inputs.

Arrays in storage dtypes are numpy arrays: ``float32``, ``float16``, and
``uint16`` bit patterns for bfloat16 (numpy has no bfloat16). Every function
follows the reference's operation order in fp32 with one rounding per
operation; the only freedom taken is the summation order of the RMS
reduction (numpy's pairwise sum).
"""

from __future__ import annotations

import numpy as np

F32 = "float32"
F16 = "float16"
BF16 = "bfloat16"
DTYPES = (F32, F16, BF16)

ROPE_STYLES = ("neox", "interleaved")


# ------------------------------------------------------------------ storage
def decode(a: np.ndarray, dtype: str) -> np.ndarray:
    """Storage array -> exact float32 values."""
    if dtype == BF16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def encode(f: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> storage dtype, round to nearest even (NaN stays NaN)."""
    f = np.asarray(f, dtype=np.float32)
    if dtype == F32:
        return f.copy()
    if dtype == F16:
        return f.astype(np.float16)
    bits = f.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        rounded[nan] = ((bits[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def storage_dtype(dtype: str) -> np.dtype:
    return {F32: np.float32, F16: np.float16, BF16: np.uint16}[dtype]


# --------------------------------------------------------------------- ops
def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, dtype: str, w_dtype: str | None = None) -> np.ndarray:
    """RMSNorm over the last axis (reference ``ako/ops/rmsnorm_ref.py:8-23``).

    ``x_c * rsqrt(mean(x_c ** 2) + eps)`` then ``* weight``, fp32, one cast.
    """
    xf = decode(x, dtype)
    wf = decode(w, w_dtype or dtype)
    sq = xf * xf  # x_c.pow(2), rounded per element
    var = np.add.reduce(sq, axis=-1, keepdims=True, dtype=np.float32) / np.float32(xf.shape[-1])
    inv = np.float32(1.0) / np.sqrt(var + np.float32(eps))  # torch.rsqrt on CPU is 1 / sqrt
    normed = xf * inv
    return encode(normed * wf, dtype)


def rmsnorm_residual(
    x: np.ndarray, r: np.ndarray, w: np.ndarray, eps: float, dtype: str, w_dtype: str | None = None
) -> tuple[np.ndarray, np.ndarray]:
    """Residual add then RMSNorm (reference ``ako/ops/rmsnorm_ref.py:26-50``).

    ``new_residual = x + residual`` in the storage dtype (one rounding), then
    ``rmsnorm(new_residual)``; returns ``(normed, new_residual)``.
    """
    if x.shape != r.shape:
        raise ValueError(f"Shape mismatch: x {x.shape} vs residual {r.shape}")
    new_res = encode(decode(x, dtype) + decode(r, dtype), dtype)
    return rmsnorm(new_res, w, eps, dtype, w_dtype), new_res


def build_rope_tables(
    seq_len: int, head_dim: int, *, base: float = 10000.0, offset: int = 0
) -> tuple[np.ndarray, np.ndarray]:
    """fp32 ``(cos, sin)`` of shape ``(seq_len, head_dim // 2)``.

    Reference ``ako/ops/rope_ref.py:20-54``: ``inv_freq = 1 / base ** (2i / D)``,
    ``freqs = outer(positions, inv_freq)``, all fp32.
    """
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even, got {head_dim}")
    half = head_dim // 2
    exponent = np.arange(0, half, dtype=np.float32) * np.float32(2.0) / np.float32(head_dim)
    inv_freq = np.float32(1.0) / np.power(np.float32(base), exponent, dtype=np.float32)
    positions = np.arange(offset, offset + seq_len, dtype=np.float32)
    freqs = np.outer(positions, inv_freq).astype(np.float32)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, style: str, dtype: str) -> np.ndarray:
    """RoPE on ``(batch, seq_len, n_heads, head_dim)`` (reference ``ako/ops/rope_ref.py:73-107``).

    neox pairs ``(i, i + D/2)``, interleaved pairs ``(2i, 2i + 1)``;
    ``[x0 * c - x1 * s, x0 * s + x1 * c]`` with each product rounded.
    """
    if style not in ROPE_STYLES:
        raise ValueError(f"Unknown RoPE style '{style}'")
    if x.ndim != 4:
        raise ValueError("Expected x of shape (batch, seq_len, n_heads, head_dim)")
    d = x.shape[-1]
    if d % 2 or cos.shape != (x.shape[1], d // 2) or sin.shape != cos.shape:
        raise ValueError("bad head_dim or table shape")
    xf = decode(x, dtype)
    c = cos.astype(np.float32)[None, :, None, :]
    s = sin.astype(np.float32)[None, :, None, :]
    if style == "neox":
        x0, x1 = xf[..., : d // 2], xf[..., d // 2 :]
        out = np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1)
    else:
        x0, x1 = xf[..., 0::2], xf[..., 1::2]
        out = np.stack([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1).reshape(xf.shape)
    return encode(out, dtype)


def swiglu(g: np.ndarray, u: np.ndarray, dtype: str) -> np.ndarray:
    """``silu(gate) * up`` in fp32 (reference ``ako/ops/swiglu_ref.py:16-32``).

    silu is ``g / (1 + exp(-g))``, the form torch's CPU kernel evaluates.
    """
    if g.shape != u.shape:
        raise ValueError(f"Shape mismatch: gate {g.shape} vs up {u.shape}")
    gf = decode(g, dtype)
    uf = decode(u, dtype)
    with np.errstate(over="ignore"):
        silu = gf / (np.float32(1.0) + np.exp(-gf))
    return encode(silu * uf, dtype)


# ---------------------------------------------------------------- compare
def ulp_distance(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """Elementwise distance in representable steps between two storage arrays."""

    def ordered(v: np.ndarray) -> np.ndarray:
        if dtype == F32:
            bits = v.astype(np.float32).view(np.int32).astype(np.int64)
            return np.where(bits < 0, -(bits & 0x7FFFFFFF), bits)
        raw = v.view(np.uint16).astype(np.int64) if dtype == F16 else v.astype(np.int64)
        return np.where(raw & 0x8000, -(raw & 0x7FFF), raw)

    return np.abs(ordered(a) - ordered(b))
