"""Parity on every cell of the benchmark configurations 1-4, on a B200.

The cells are the configurations' own shapes and distributions:

* config 1: RMSNorm fp32, x [4, 512, 4096] ~ N(0, 1), weight ~ N(1, 0.1), eps 1e-6;
* config 2: fused residual RMSNorm, bf16 and fp16, H in {2048, 4096, 8192,
  16384} x M in {1, 32, 512, 8192, 32768} (40 cells), x and residual
  ~ N(0, 1), weight ~ N(1, 0.1), eps 1e-5;
* config 3: RoPE (neox), bf16 and fp16, q [B, S, 32, 128] and k [B, S, 8, 128],
  B in {1, 8, 32} x S in {1 (position 2047), 512, 4096} (18 cells x q, k),
  the fp32 table of 8192 positions sliced per call;
* config 4: SwiGLU, bf16 and fp16, F in {5632, 11008, 14336} x M in {1, 64,
  2048, 16384}, separate [M, F] operands and the packed [M, 2F] halves
  (48 cells), gate and up ~ N(0, 2).

Inputs are seeded per cell and generated on the device; outputs are compared
with the C oracle on every row of cells that move at most 64 MB, and on a
spread of rows (first, last, and seeded random ones) of larger cells. The
gates: RMSNorm bit for bit against the fixed-order model and within the
reference gate of the reference-order oracle (config 1 within 4 ulp
elementwise, the north star's fp32 bound); the rounded residual and RoPE bit
for bit; SwiGLU within 2 ulp.

With ``AKO_B200_ULP_REPORT=<path>`` each cell appends one JSON line with its
maximum elementwise ulp distance from the reference-order oracle.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from ako_b200 import kernels
from helpers import TORCH_DTYPE, assert_parity, check_rmsnorm, to_numpy, to_torch
from oracle import ako_oracle as O
from oracle import c_oracle as C

pytestmark = pytest.mark.gpu

ALL_ROWS_BYTES = 64 << 20
SAMPLE_ROWS = 192


def _report(cell: str, **fields) -> None:
    path = os.environ.get("AKO_B200_ULP_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"cell": cell, **fields}) + "\n")


def _rows(m: int, moved: int, seed: int) -> list[int]:
    if moved <= ALL_ROWS_BYTES or m <= SAMPLE_ROWS:
        return list(range(m))
    rng = np.random.default_rng(seed)
    return sorted({0, 1, m // 2, m - 2, m - 1, *rng.choice(m, SAMPLE_ROWS - 5, replace=False).tolist()})


def _randn(shape, gen: torch.Generator, device, dtype, mean: float = 0.0, std: float = 1.0) -> torch.Tensor:
    return (torch.randn(*shape, generator=gen, device=device) * std + mean).to(dtype)


def _max_ulp(ref: np.ndarray, out: np.ndarray, dtype: str) -> int:
    return int(O.ulp_distance(ref, out, dtype).max()) if ref.size else 0


# ------------------------------------------------------------------ config 1
def test_config1_rmsnorm_fp32(cuda_device) -> None:
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((4, 512, 4096), dtype=np.float32))
    w = rng.standard_normal(4096, dtype=np.float32) * np.float32(0.1) + np.float32(1.0)
    y = kernels.rmsnorm_cuda_sm100(to_torch(x, O.F32, cuda_device), to_torch(w, O.F32, cuda_device), 1e-6)
    out = to_numpy(y).reshape(-1, 4096)
    x2 = x.reshape(-1, 4096)
    check_rmsnorm(x2, None, w, 1e-6, O.F32, out, what="config 1")
    ulp = _max_ulp(C.rmsnorm(x2, w, 1e-6, O.F32), out, O.F32)
    _report("config1 rmsnorm fp32 [4,512,4096]", max_ulp=ulp)
    assert ulp <= 4, f"config 1: {ulp} ulp elementwise"


# ------------------------------------------------------------------ config 2
CONFIG2 = [(dt, h, m) for dt in (O.BF16, O.F16) for h in (2048, 4096, 8192, 16384) for m in (1, 32, 512, 8192, 32768)]


@pytest.mark.parametrize("dtype, h, m", CONFIG2, ids=[f"{d}-H{h}-M{m}" for d, h, m in CONFIG2])
def test_config2_rmsnorm_residual(cuda_device, dtype: str, h: int, m: int) -> None:
    tdt = TORCH_DTYPE[dtype]
    gen = torch.Generator(device=cuda_device).manual_seed(h * 100003 + m)
    x = _randn((m, h), gen, cuda_device, tdt)
    r = _randn((m, h), gen, cuda_device, tdt)
    w = _randn((h,), gen, cuda_device, tdt, 1.0, 0.1)
    y, ro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
    sel = _rows(m, 4 * m * h * 2, m + h)
    xs, rs, wn = to_numpy(x[sel]), to_numpy(r[sel]), to_numpy(w)
    ys = to_numpy(y[sel])
    check_rmsnorm(xs, rs, wn, 1e-5, dtype, ys, to_numpy(ro[sel]), what=f"config 2 {dtype} H{h} M{m}")
    _report(f"config2 rmsnorm_residual {dtype} H{h} M{m}", rows_checked=len(sel),
            max_ulp=_max_ulp(C.rmsnorm_residual(xs, rs, wn, 1e-5, dtype)[0], ys, dtype))


# ------------------------------------------------------------------ config 3
CONFIG3 = [(dt, b, s) for dt in (O.BF16, O.F16) for b in (1, 8, 32) for s in (1, 512, 4096)]
_TABLES: dict[str, tuple[np.ndarray, np.ndarray]] = {}


def _tables() -> tuple[np.ndarray, np.ndarray]:
    if "t" not in _TABLES:
        _TABLES["t"] = O.build_rope_tables(8192, 128)
    return _TABLES["t"]


@pytest.mark.parametrize("dtype, b, s", CONFIG3, ids=[f"{d}-B{b}-S{s}" for d, b, s in CONFIG3])
def test_config3_rope_q_and_k(cuda_device, dtype: str, b: int, s: int) -> None:
    tdt = TORCH_DTYPE[dtype]
    cos_full, sin_full = _tables()
    off = 2047 if s == 1 else 0
    cos_d = to_torch(cos_full, O.F32, cuda_device)[off:off + s]
    sin_d = to_torch(sin_full, O.F32, cuda_device)[off:off + s]
    gen = torch.Generator(device=cuda_device).manual_seed(b * 10007 + s)
    q = _randn((b, s, 32, 128), gen, cuda_device, tdt)
    k = _randn((b, s, 8, 128), gen, cuda_device, tdt)
    for name, t in (("q", q), ("k", k)):
        y = kernels.rope_cuda_sm100(t, cos_d, sin_d, "neox")
        sel = _rows(s, 2 * t.numel() * 2, b + s)
        ref = C.rope(to_numpy(t[:, sel]), cos_full[off:off + s][sel], sin_full[off:off + s][sel], "neox", dtype)
        out = to_numpy(y[:, sel])
        np.testing.assert_array_equal(out, ref, err_msg=f"config 3 {name} {dtype} B{b} S{s}")
        _report(f"config3 rope {name} {dtype} B{b} S{s}", positions_checked=len(sel) * b, max_ulp=0)
    # the fused pair gives the same bytes in one launch
    qo, ko = kernels.rope_qk_cuda_sm100(q, k, cos_d, sin_d, "neox")
    assert torch.equal(qo, kernels.rope_cuda_sm100(q, cos_d, sin_d, "neox"))
    assert torch.equal(ko, kernels.rope_cuda_sm100(k, cos_d, sin_d, "neox"))


# ------------------------------------------------------------------ config 4
CONFIG4 = [(dt, f, m, packed) for dt in (O.BF16, O.F16) for f in (5632, 11008, 14336) for m in (1, 64, 2048, 16384)
           for packed in (False, True)]


@pytest.mark.parametrize("dtype, f, m, packed", CONFIG4,
                         ids=[f"{d}-F{f}-M{m}-{'packed' if p else 'separate'}" for d, f, m, p in CONFIG4])
def test_config4_swiglu(cuda_device, dtype: str, f: int, m: int, packed: bool) -> None:
    tdt = TORCH_DTYPE[dtype]
    gen = torch.Generator(device=cuda_device).manual_seed(f * 7919 + m * 2 + int(packed))
    if packed:
        both = _randn((m, 2 * f), gen, cuda_device, tdt, 0.0, 2.0)
        g, u = both[:, :f], both[:, f:]
    else:
        g = _randn((m, f), gen, cuda_device, tdt, 0.0, 2.0)
        u = _randn((m, f), gen, cuda_device, tdt, 0.0, 2.0)
    y = kernels.swiglu_cuda_sm100(g, u)
    sel = _rows(m, 3 * m * f * 2, f + m)
    ref = C.swiglu(to_numpy(g[sel]), to_numpy(u[sel]), dtype)
    out = to_numpy(y[sel])
    assert_parity(ref, out, dtype, "swiglu", f"config 4 {dtype} F{f} M{m} packed={packed}")
    _report(f"config4 swiglu {dtype} F{f} M{m} {'packed' if packed else 'separate'}", rows_checked=len(sel),
            max_ulp=_max_ulp(ref, out, dtype))
