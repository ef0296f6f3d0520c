"""Conversions between torch tensors and the oracle's numpy storage arrays,
seeded input generation, and the tolerance gates every parity test uses."""

from __future__ import annotations

import math

import numpy as np
import torch

from oracle import ako_oracle as O

TORCH_DTYPE = {O.F32: torch.float32, O.F16: torch.float16, O.BF16: torch.bfloat16}
NAME = {v: k for k, v in TORCH_DTYPE.items()}

#: Elementwise ulp bounds against the reference / oracle.
#: 16-bit outputs: the budget the hot path is held to (2 ulp).
#: fp32: rmsnorm's sum of H squares may be ordered differently from the
#: reference's; two pairwise orders differ by at most ~log2(H)/2 ulp of the
#: sum, which moves rsqrt by half of that, plus three roundings; 8 ulp covers
#: H <= 65536. RoPE is bit-exact; SwiGLU fp32 differs by the exp
#: implementations (<= 2 ulp each) through one division and one product.
ULP_16 = 2
ULP_F32 = {"rmsnorm": 8, "rmsnorm_residual": 8, "rope": 0, "swiglu": 6}
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
