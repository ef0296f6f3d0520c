"""Conversions between torch tensors and the oracle's numpy storage arrays,
seeded input generation, and the tolerance gates every parity test uses."""

from __future__ import annotations

import math

import numpy as np
import torch

from oracle import ako_oracle as O
from oracle import c_oracle as C

TORCH_DTYPE = {O.F32: torch.float32, O.F16: torch.float16, O.BF16: torch.bfloat16}
NAME = {v: k for k, v in TORCH_DTYPE.items()}

#: Elementwise ulp bounds against the reference / oracle.
#: 16-bit outputs: the budget the hot path is held to (2 ulp).
#: fp32 RMSNorm: the kernels sum a row's squares in their own fixed order
#: (checked bit for bit against the C model of it), the reference in torch's
#: CPU order, which depends on the CPU's vector width. Two orders of the same
#: sum differ by a few ulp of the sum, rsqrt halves that, and two roundings
#: follow. Measured (fixed order against the reference): at most 4 ulp on
#: config 1's [4, 512, 4096] cell and on rows of 2048-65536 elements against
#: the reference-order oracle, and 6 ulp on 5 of 67 million elements of a
#: [8, 2048, 4096] batch against torch itself; hence 6. AKO's own report
#: (relative to max|ref|) stays within its 4-ulp target (AKO_ULPS).
#: RoPE is bit-exact. SwiGLU fp32 differs by the exp implementations (CUDA's
#: expf within 2 ulp, the reference's within 1) through a division and a
#: product.
ULP_16 = 2
ULP_F32 = {"rmsnorm": 6, "rmsnorm_residual": 6, "rope": 0, "swiglu": 6}
#: AKO's own report (error_in_ulps, error relative to max|ref|): 2 / 4 ulp.
AKO_ULPS = {O.F32: 4.0, O.F16: 2.0, O.BF16: 2.0}


def to_torch(a: np.ndarray, dtype: str, device: torch.device | str = "cpu") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype == O.BF16:
        t = t.view(torch.int16).view(torch.bfloat16)
    return t.to(device)


def to_numpy(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def normal(rng: np.random.Generator, shape, mean: float, std: float, dtype: str) -> np.ndarray:
    """Seeded N(mean, std) in the storage dtype."""
    return O.encode((rng.standard_normal(shape, dtype=np.float32) * np.float32(std) + np.float32(mean)), dtype)


def ako_error_in_ulps(ref: np.ndarray, out: np.ndarray, dtype: str) -> float:
    """AKO's ``error_in_ulps``: max abs error over the spacing at max|ref|."""
    rf, of = O.decode(ref, dtype), O.decode(out, dtype)
    mag = float(np.abs(rf).max()) if rf.size else 0.0
    eps = {O.F32: 2.0**-23, O.F16: 2.0**-10, O.BF16: 2.0**-7}[dtype]
    tiny = {O.F32: 2.0**-126, O.F16: 2.0**-14, O.BF16: 2.0**-126}[dtype]
    spacing = tiny if mag < tiny else math.ldexp(1.0, math.floor(math.log2(mag))) * eps
    err = float(np.abs(rf.astype(np.float64) - of.astype(np.float64)).max()) if rf.size else 0.0
    return err / spacing


def ako_error_budget(ref: np.ndarray, dtype: str) -> float:
    """AKO's ``error_budget``: ``1e-5 + rtol(dtype) * max|ref|``."""
    rtol = {O.F32: 1.3e-6, O.F16: 1e-3, O.BF16: 1.6e-2}[dtype]
    rf = O.decode(ref, dtype)
    return 1e-5 + rtol * (float(np.abs(rf).max()) if rf.size else 0.0)


def assert_parity(ref: np.ndarray, out: np.ndarray, dtype: str, op: str, what: str = "") -> None:
    """The gate: AKO's budget and ulp report, plus the elementwise ulp bound."""
    assert ref.shape == out.shape, f"{what}: shape {out.shape} != {ref.shape}"
    if ref.size == 0:
        return
    d = O.ulp_distance(ref, out, dtype)
    bound = ULP_16 if dtype != O.F32 else ULP_F32[op]
    rf, of = O.decode(ref, dtype), O.decode(out, dtype)
    err = float(np.abs(rf.astype(np.float64) - of.astype(np.float64)).max())
    assert err <= ako_error_budget(ref, dtype), f"{what}: max_error {err} > AKO budget"
    assert ako_error_in_ulps(ref, out, dtype) <= AKO_ULPS[dtype], f"{what}: AKO ulps"
    assert int(d.max()) <= bound, f"{what}: elementwise ulp {int(d.max())} > {bound} ({int((d > 0).sum())} differ)"


def whole_vectors(h: int, dtype: str) -> bool:
    """Rows of ``h`` elements are whole 16-byte vectors (the vector kernels' rows)."""
    return (h * (4 if dtype == O.F32 else 2)) % 16 == 0


def check_rmsnorm(x: np.ndarray, r: np.ndarray | None, w: np.ndarray, eps: float, dtype: str, y: np.ndarray,
                  ro: np.ndarray | None = None, *, w_dtype: str | None = None, exact: bool | None = None,
                  what: str = "") -> None:
    """RMSNorm (``r`` None) or fused residual RMSNorm outputs of the CUDA path.

    * Against the reference-order oracle: the parity gate, and the rounded
      residual bit for bit.
    * ``exact`` (default: rows of whole 16-byte vectors, the vector kernels'
      rows): bit for bit against the C model of the kernels' fixed summation
      order, which depends on the row width only.
    """
    if r is None:
        ref = C.rmsnorm(x, w, eps, dtype, w_dtype)
        assert_parity(ref, y, dtype, "rmsnorm", what)
    else:
        ref, ro_ref = C.rmsnorm_residual(x, r, w, eps, dtype, w_dtype)
        np.testing.assert_array_equal(ro, ro_ref, err_msg=f"{what}: residual")
        assert_parity(ref, y, dtype, "rmsnorm_residual", what)
    if exact is None:
        exact = whole_vectors(x.shape[-1], dtype)
    if exact:
        model = C.rmsnorm_fixed_order(x, r, w, eps, dtype, w_dtype)
        y_model = model if r is None else model[0]
        if not np.array_equal(y, y_model):
            d = O.ulp_distance(y_model, y, dtype)
            raise AssertionError(f"{what}: differs from the fixed-order model in {int((d > 0).sum())} elements "
                                 f"(max {int(d.max())} ulp)")
