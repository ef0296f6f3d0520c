"""Parity of the sm_100a kernels with the reference, on a B200.

Every call goes through the C ABI (``libako_b200.so``) via the KernelFn
wrappers. Outputs are compared with the golden vectors the reference produced
and with the CPU oracle on the same seeded inputs, under the gates of
``helpers.assert_parity``: AKO's budget, AKO's ulp report (2 ulp for 16-bit,
4 for fp32) and an elementwise ulp bound. The rounded residual and RoPE are
compared bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import golden_data as gd
from ako_b200 import _native, kernels
from helpers import TORCH_DTYPE, assert_parity, check_rmsnorm, normal, to_numpy, to_torch
from oracle import ako_oracle as O
from oracle import c_oracle as C

pytestmark = pytest.mark.gpu

DTYPES = (O.F32, O.F16, O.BF16)


def dev() -> torch.device:
    return torch.device("cuda", 0)


# ------------------------------------------------------------------ golden
@pytest.mark.parametrize("case", gd.cases(), ids=[c["name"] for c in gd.cases()])
def test_golden_vectors(cuda_device, case) -> None:
    dt = case["dtype"]
    t = lambda k: to_torch(gd.arr(case, k), dt if k not in ("cos", "sin") else O.F32, cuda_device)  # noqa: E731
    op = case["op"]
    if op == "rmsnorm":
        out = {"y": kernels.rmsnorm_cuda_sm100(t("x"), t("w"), case["eps"])}
    elif op == "rmsnorm_residual":
        y, ro = kernels.rmsnorm_residual_cuda_sm100(t("x"), t("r"), t("w"), case["eps"])
        out = {"y": y, "ro": ro}
    elif op == "rope":
        out = {"y": kernels.rope_cuda_sm100(t("x"), t("cos"), t("sin"), case["style"])}
    else:
        out = {"y": kernels.swiglu_cuda_sm100(t("g"), t("u"))}
    torch.cuda.synchronize()
    if "ro" in out:
        np.testing.assert_array_equal(to_numpy(out["ro"]), gd.arr(case, "ro"))
    if op == "rope":
        np.testing.assert_array_equal(to_numpy(out["y"]), gd.arr(case, "y"))
    assert_parity(gd.arr(case, "y"), to_numpy(out["y"]), dt, op, case["name"])


# ----------------------------------------------------------------- rmsnorm
HIDDEN = (1, 2, 7, 64, 100, 256, 512, 1000, 1024, 2048, 4096, 5120, 8192, 8448, 11008, 16384, 32768, 65536)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("h", HIDDEN)
def test_rmsnorm_widths(cuda_device, dtype: str, h: int) -> None:
    rng = np.random.default_rng(h)
    rows = 5 if h <= 16384 else 2
    x = normal(rng, (rows, h), 0, 1, dtype)
    r = normal(rng, (rows, h), 0, 1, dtype)
    w = normal(rng, (h,), 1, 0.1, dtype)
    y = kernels.rmsnorm_cuda_sm100(to_torch(x, dtype, cuda_device), to_torch(w, dtype, cuda_device), 1e-6)
    check_rmsnorm(x, None, w, 1e-6, dtype, to_numpy(y), what=f"rmsnorm h={h}")
    y, ro = kernels.rmsnorm_residual_cuda_sm100(
        to_torch(x, dtype, cuda_device), to_torch(r, dtype, cuda_device), to_torch(w, dtype, cuda_device), 1e-5
    )
    check_rmsnorm(x, r, w, 1e-5, dtype, to_numpy(y), to_numpy(ro), what=f"residual h={h}")


@pytest.mark.parametrize("rows", [1, 3, 4, 5, 127, 1000])
def test_rmsnorm_row_counts(cuda_device, rows: int) -> None:
    """Warp-per-row CTAs hold four rows; partial last CTAs must be exact."""
    for h in (256, 1024, 4096):
        rng = np.random.default_rng(rows * h)
        x = normal(rng, (rows, h), 0, 1, O.BF16)
        r = normal(rng, (rows, h), 0, 1, O.BF16)
        w = normal(rng, (h,), 1, 0.1, O.BF16)
        y, ro = kernels.rmsnorm_residual_cuda_sm100(*(to_torch(a, O.BF16, cuda_device) for a in (x, r, w)), 1e-5)
        check_rmsnorm(x, r, w, 1e-5, O.BF16, to_numpy(y), to_numpy(ro), what=f"rows={rows} h={h}")


@pytest.mark.parametrize("dtype", DTYPES)
def test_rmsnorm_strided_and_misaligned_rows(cuda_device, dtype: str) -> None:
    """Row-strided views run in place; unaligned ones take the scalar kernel."""
    rng = np.random.default_rng(7)
    base = to_torch(normal(rng, (6, 4100), 0, 1, dtype), dtype, cuda_device)
    w = to_torch(normal(rng, (4096,), 1, 0.1, dtype), dtype, cuda_device)
    for x in (base[:, :4096], base[:, 1:4097], base[:, 4:4100]):
        y = kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
        ref = C.rmsnorm(to_numpy(x), to_numpy(w), 1e-6, dtype)
        assert_parity(ref, to_numpy(y), dtype, "rmsnorm", "strided")


@pytest.mark.parametrize("dtype", DTYPES)
def test_rmsnorm_narrow_rows_in_bulk(cuda_device, dtype: str) -> None:
    """Narrow rows in many rows take a warp per row with 4 or 8 vectors a
    thread (65-224 vectors, from 8192 or 16384 rows): plain and fused against
    the oracle on a sample of rows, including partial last CTAs."""
    vec = 4 if dtype == O.F32 else 8
    g = torch.Generator(device=cuda_device).manual_seed(29)
    tdt = TORCH_DTYPE[dtype]
    for nvec in (65, 96, 128, 160, 224):
        h = nvec * vec
        rows = 16387
        x = torch.randn(rows, h, generator=g, device=cuda_device).to(tdt)
        r = torch.randn(rows, h, generator=g, device=cuda_device).to(tdt)
        w = (torch.randn(h, generator=g, device=cuda_device) * 0.1 + 1).to(tdt)
        sel = list(range(0, rows, 1021)) + [rows - 3, rows - 2, rows - 1]
        y = kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
        assert_parity(C.rmsnorm(to_numpy(x[sel]), to_numpy(w), 1e-6, dtype), to_numpy(y[sel]), dtype, "rmsnorm",
                      f"narrow h={h}")
        y, ro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
        y_ref, ro_ref = C.rmsnorm_residual(to_numpy(x[sel]), to_numpy(r[sel]), to_numpy(w), 1e-5, dtype)
        np.testing.assert_array_equal(to_numpy(ro[sel]), ro_ref)
        assert_parity(y_ref, to_numpy(y[sel]), dtype, "rmsnorm_residual", f"narrow h={h}")


@pytest.mark.parametrize("dtype", DTYPES)
def test_rmsnorm_generic_weight_alignments(cuda_device, dtype: str) -> None:
    """The any-width kernel reads a weight of the row's dtype through aligned
    16-byte blocks shifted by the weight's misalignment within the row body:
    every misalignment a weight view can have, ragged and aligned widths,
    plain and fused, against the oracle (the first and last body vectors of a
    view whose blocks would reach outside it read element by element)."""
    rng = np.random.default_rng(41)
    vec = 4 if dtype == O.F32 else 8
    for h in (4100, 4096, 1000, 37):
        rows = 6
        x = normal(rng, (rows, h), 0, 1, dtype)
        r = normal(rng, (rows, h), 0, 1, dtype)
        wbase = normal(rng, (h + 2 * vec,), 1, 0.1, dtype)
        xt, rt = to_torch(x, dtype, cuda_device), to_torch(r, dtype, cuda_device)
        wt_base = to_torch(wbase, dtype, cuda_device)
        for off in range(vec + 1):
            w = wbase[off:off + h]
            wt = wt_base[off:off + h]
            y = kernels.rmsnorm_cuda_sm100(xt, wt, 1e-6)
            assert_parity(C.rmsnorm(x, w, 1e-6, dtype), to_numpy(y), dtype, "rmsnorm", f"h={h} weight offset {off}")
            y, ro = kernels.rmsnorm_residual_cuda_sm100(xt, rt, wt, 1e-5)
            y_ref, ro_ref = C.rmsnorm_residual(x, r, w, 1e-5, dtype)
            np.testing.assert_array_equal(to_numpy(ro), ro_ref)
            assert_parity(y_ref, to_numpy(y), dtype, "rmsnorm_residual", f"h={h} weight offset {off}")


@pytest.mark.parametrize("dtype", DTYPES)
def test_rmsnorm_generic_warp_and_cta_per_row(cuda_device, dtype: str) -> None:
    """The any-width kernel with a warp per row (four rows per CTA, so row
    counts that leave the last CTA part-empty) and with a CTA per row, forced
    through the measurement build: ragged widths, rows starting off 16-byte
    boundaries (a column slice of a wider tensor), fused and plain, a weight
    of the row's dtype and an fp32 one, against the oracle."""
    rng = np.random.default_rng(43)
    with _native.measurement() as lib:
        try:
            for tpr in (32, 256):
                assert lib.ako_b200_rmsnorm_set_generic(tpr) == 0
                for h in (1, 7, 37, 1001, 2047, 4100):
                    for rows, shift in ((1, 0), (5, 0), (9, 1), (6, 3)):
                        xb = normal(rng, (rows, h + shift), 0, 1, dtype)
                        rb = normal(rng, (rows, h + shift), 0, 1, dtype)
                        x, r = xb[:, shift:], rb[:, shift:]
                        w = normal(rng, (h,), 1, 0.1, dtype)
                        w32 = normal(rng, (h,), 1, 0.1, O.F32)
                        xt = to_torch(xb, dtype, cuda_device)[:, shift:]
                        rt = to_torch(rb, dtype, cuda_device)[:, shift:]
                        wt = to_torch(w, dtype, cuda_device)
                        what = f"{tpr} threads/row h={h} rows={rows} shift={shift}"
                        y = kernels.rmsnorm_cuda_sm100(xt, wt, 1e-6)
                        assert_parity(C.rmsnorm(x, w, 1e-6, dtype), to_numpy(y), dtype, "rmsnorm", what)
                        y, ro = kernels.rmsnorm_residual_cuda_sm100(xt, rt, wt, 1e-5)
                        y_ref, ro_ref = C.rmsnorm_residual(x, r, w, 1e-5, dtype)
                        np.testing.assert_array_equal(to_numpy(ro), ro_ref)
                        assert_parity(y_ref, to_numpy(y), dtype, "rmsnorm_residual", what)
                        y = kernels.rmsnorm_cuda_sm100(xt, to_torch(w32, O.F32, cuda_device), 1e-6)
                        assert_parity(C.rmsnorm(x, w32, 1e-6, dtype, O.F32), to_numpy(y), dtype, "rmsnorm",
                                      what + " fp32 weight")
        finally:
            lib.ako_b200_rmsnorm_set_generic(0)


@pytest.mark.parametrize("dtype", (O.F16, O.BF16))
def test_rmsnorm_fp32_weight(cuda_device, dtype: str) -> None:
    rng = np.random.default_rng(11)
    x = normal(rng, (8, 4096), 0, 1, dtype)
    w = normal(rng, (4096,), 1, 0.1, O.F32)
    y = kernels.rmsnorm_cuda_sm100(to_torch(x, dtype, cuda_device), to_torch(w, O.F32, cuda_device), 1e-6)
    assert_parity(C.rmsnorm(x, w, 1e-6, dtype, O.F32), to_numpy(y), dtype, "rmsnorm", "fp32 weight")


def test_every_rmsnorm_launch_shape(cuda_device) -> None:
    """All built (cluster, threads per row slice, vectors per thread) shapes,
    forced through the measurement build, give the fixed summation order's
    bits (so every shape gives the same bits), on rows one vector per CTA
    slice short of full and, for clusters, on rows of whole 32-vector groups
    per slice."""
    rng = np.random.default_rng(5)
    single = [(32, 1), (32, 2), (32, 4), (32, 8), (64, 2), (64, 4), (64, 8), (128, 1), (128, 2), (128, 4),
              (128, 8), (256, 1), (256, 2), (256, 4), (256, 8), (512, 1), (512, 2), (512, 4), (512, 8),
              (1024, 1), (1024, 2), (1024, 4), (1024, 8), (96, 2), (96, 4), (160, 2), (160, 4), (192, 2), (192, 4),
              (224, 2), (224, 4), (320, 2), (320, 4), (384, 2), (384, 4), (448, 2), (448, 4), (640, 2), (640, 4),
              (768, 2), (768, 4), (896, 2), (896, 4)]
    split = [(64, 4), (128, 2), (128, 4), (256, 2), (256, 4), (512, 2), (512, 4), (1024, 1), (1024, 2)]
    shapes = [(1, t, n) for t, n in single] + [(c, t, n) for c in (2, 4, 8) for t, n in split]
    with _native.measurement() as lib:
        try:
            for dtype in (O.BF16, O.F32):
                vec = 8 if dtype == O.BF16 else 4
                for cl, tpr, nv in shapes:
                    # one vector short per CTA slice exercises the mask; a cluster
                    # splits rows only into whole 32-vector groups per slice
                    nvec = tpr * nv - 1 if cl == 1 else (tpr * nv - 32 if tpr * nv > 32 else 32)
                    h = cl * nvec * vec
                    if h < vec or h > 65536:
                        continue
                    rows = 9 if h <= 16384 else 3
                    x = normal(rng, (rows, h), 0, 1, dtype)
                    r = normal(rng, (rows, h), 0, 1, dtype)
                    w = normal(rng, (h,), 1, 0.1, dtype)
                    assert lib.ako_b200_rmsnorm_set_launch(cl, tpr, nv) == 0
                    args = (to_torch(a, dtype, cuda_device) for a in (x, r, w))
                    y, ro = kernels.rmsnorm_residual_cuda_sm100(*args, 1e-5)
                    check_rmsnorm(x, r, w, 1e-5, dtype, to_numpy(y), to_numpy(ro), what=f"shape {cl}x{tpr}x{nv} h={h}")
                    y1 = kernels.rmsnorm_cuda_sm100(to_torch(x, dtype, cuda_device), to_torch(w, dtype, cuda_device),
                                                    1e-6)
                    check_rmsnorm(x, None, w, 1e-6, dtype, to_numpy(y1), what=f"shape {cl}x{tpr}x{nv}")
                    if dtype == O.BF16:
                        # a weight of another dtype takes the kernel's second weight path
                        w32 = normal(rng, (h,), 1, 0.1, O.F32)
                        y2 = kernels.rmsnorm_cuda_sm100(to_torch(x, dtype, cuda_device),
                                                        to_torch(w32, O.F32, cuda_device), 1e-6)
                        check_rmsnorm(x, None, w32, 1e-6, dtype, to_numpy(y2), w_dtype=O.F32,
                                      what=f"fp32 weight, shape {cl}x{tpr}x{nv}")
        finally:
            lib.ako_b200_rmsnorm_set_launch(0, 0, 0)


@pytest.mark.parametrize("dtype", DTYPES)
def test_rmsnorm_fitted_thread_counts(cuda_device, dtype: str) -> None:
    """Common widths that are not powers of two (2560 ... 13824) with enough
    rows for the throughput table, which fits the thread count to the row
    (e.g. 320 threads x 2 vectors for 5120 bf16 elements); plain and fused,
    against the oracle, with ragged widths next to them."""
    rng = np.random.default_rng(23)
    for h in (2560, 3072, 3584, 5120, 6144, 7168, 12288, 13824, 5128, 12296, 4608, 9216, 11264):
        rows = 600
        x = normal(rng, (rows, h), 0, 1, dtype)
        r = normal(rng, (rows, h), 0, 1, dtype)
        w = normal(rng, (h,), 1, 0.1, dtype)
        xt, rt, wt = (to_torch(a, dtype, cuda_device) for a in (x, r, w))
        y, ro = kernels.rmsnorm_residual_cuda_sm100(xt, rt, wt, 1e-5)
        check_rmsnorm(x, r, w, 1e-5, dtype, to_numpy(y), to_numpy(ro), what=f"fitted h={h}")
        y1 = kernels.rmsnorm_cuda_sm100(xt, wt, 1e-6)
        check_rmsnorm(x, None, w, 1e-6, dtype, to_numpy(y1), what=f"fitted h={h}")


@pytest.mark.parametrize("dtype", DTYPES)
def test_staged_rmsnorm_matches_oracle(cuda_device, dtype: str) -> None:
    """The persistent bulk-copy kernel (forced through the measurement
    build): every stage count and CTA density, rows fewer than CTAs, many rows
    per CTA, strided rows, fp32 weights. Both outputs equal the row-resident
    kernel's and the fixed-order model's bit for bit; no bounded wait ran
    out."""
    rng = np.random.default_rng(31)
    vec = 8 if dtype != O.F32 else 4
    with _native.measurement() as lib:
        _staged_cases(lib, cuda_device, rng, dtype, vec)


def _staged_cases(lib, cuda_device, rng, dtype, vec) -> None:
    try:
        for h in (vec, 256, 1000 if dtype == O.F32 else 1000 - 1000 % vec, 2048, 4096, 8192, 16384):
            if h % vec or h * (4 if dtype == O.F32 else 2) > 32768:
                continue
            for rows, stages, ctas in ((1, 4, 2), (3, 1, 1), (300, 2, 1), (700, 8, 4), (1500, 3, 2)):
                if rows * h > 4_000_000:
                    rows = max(1, 4_000_000 // h)
                x = normal(rng, (rows, h), 0, 1, dtype)
                r = normal(rng, (rows, h), 0, 1, dtype)
                w = normal(rng, (h,), 1, 0.1, dtype)
                xt, rt, wt = (to_torch(a, dtype, cuda_device) for a in (x, r, w))
                assert lib.ako_b200_rmsnorm_set_staging(2, stages, ctas) == 0
                y_s, ro_s = kernels.rmsnorm_residual_cuda_sm100(xt, rt, wt, 1e-5)
                y1_s = kernels.rmsnorm_cuda_sm100(xt, wt, 1e-6)
                assert lib.ako_b200_rmsnorm_set_staging(1, 0, 0) == 0
                y_r, ro_r = kernels.rmsnorm_residual_cuda_sm100(xt, rt, wt, 1e-5)
                y1_r = kernels.rmsnorm_cuda_sm100(xt, wt, 1e-6)
                assert torch.equal(ro_s, ro_r) and torch.equal(y_s, y_r) and torch.equal(y1_s, y1_r), (h, rows)
                check_rmsnorm(x, r, w, 1e-5, dtype, to_numpy(y_s), to_numpy(ro_s), what=f"staged h={h} rows={rows}")
                check_rmsnorm(x, None, w, 1e-6, dtype, to_numpy(y1_s), what=f"staged h={h}")
        # strided rows and an fp32 weight through the staged path
        base = to_torch(normal(rng, (64, 4096 + 64), 0, 1, dtype), dtype, cuda_device)
        xs = base[:, 64:]
        wf = to_torch(normal(rng, (4096,), 1, 0.1, O.F32), O.F32, cuda_device)
        assert lib.ako_b200_rmsnorm_set_staging(2, 4, 2) == 0
        y = kernels.rmsnorm_cuda_sm100(xs, wf, 1e-6)
        check_rmsnorm(to_numpy(xs), None, to_numpy(wf), 1e-6, dtype, to_numpy(y), w_dtype=O.F32,
                      what="staged strided")
        torch.cuda.synchronize()
        assert _native.take_device_status() == 0
    finally:
        lib.ako_b200_rmsnorm_set_staging(0, 0, 0)


BATCH_WIDTHS = [(O.BF16, h) for h in (2048, 4096, 5120, 8192, 11008, 14336, 16384, 32768, 65536)] + [
    (O.F16, 65536), (O.F16, 4096), (O.F32, 4096), (O.F32, 16384), (O.F32, 32768)]


@pytest.mark.parametrize("dtype, h", BATCH_WIDTHS, ids=[f"{d}-{h}" for d, h in BATCH_WIDTHS])
def test_rmsnorm_bits_do_not_depend_on_batch_size(cuda_device, dtype: str, h: int) -> None:
    """The same rows normalized in batches of 1 to 8192 rows, which the
    built-in choice runs on different kernels and launch shapes (clusters for
    decode, latency shapes, the throughput table, the staged and chunked
    persistent kernels), give identical bits, plain and fused; and they equal
    the fixed-order model."""
    tdt = TORCH_DTYPE[dtype]
    g = torch.Generator(device=cuda_device).manual_seed(h)
    full = max(1, min(8192, (1 << 27) // h))
    x = torch.randn(full, h, generator=g, device=cuda_device).to(tdt)
    r = torch.randn(full, h, generator=g, device=cuda_device).to(tdt)
    w = (torch.randn(h, generator=g, device=cuda_device) * 0.1 + 1).to(tdt)
    y_full = kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
    yr_full, ro_full = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
    for n in (1, 2, 8, 9, 32, 33, 64, 65, 148, 512, 513, 1024, 2048, 4096):
        if n >= full:
            continue
        assert torch.equal(kernels.rmsnorm_cuda_sm100(x[:n], w, 1e-6), y_full[:n]), (dtype, h, n)
        yr, ro = kernels.rmsnorm_residual_cuda_sm100(x[:n], r[:n], w, 1e-5)
        assert torch.equal(yr, yr_full[:n]) and torch.equal(ro, ro_full[:n]), (dtype, h, n)
    sel = [0, full // 2, full - 1]
    xs, rs, wn = to_numpy(x[sel]), to_numpy(r[sel]), to_numpy(w)
    check_rmsnorm(xs, None, wn, 1e-6, dtype, to_numpy(y_full[sel]), what=f"batch h={h}")
    check_rmsnorm(xs, rs, wn, 1e-5, dtype, to_numpy(yr_full[sel]), to_numpy(ro_full[sel]), what=f"batch h={h}")


def test_bounded_wait_expiry_is_reported_and_never_silent(cuda_device) -> None:
    """A persistent kernel whose bounded wait for a bulk copy runs out fills
    the rows it could not produce with NaN and records the expiry; every
    later call of that library is refused until the status is taken. Forced
    through the measurement build with a wait limit of 0 polls: the waits
    give up at once while the copies themselves still land, and the kernel
    drains them before it exits. The product library's status is separate
    and stays clear."""
    g = torch.Generator(device=cuda_device).manual_seed(41)
    bf = torch.bfloat16
    cases = [(2, 64, 4096, False), (2, 64, 4096, True), (3, 9, 65536, False)]  # staged plain, staged fused, chunked
    with _native.measurement() as lib:
        try:
            for mode, rows, h, fused in cases:
                x = torch.randn(rows, h, generator=g, device=cuda_device).to(bf)
                r = torch.randn(rows, h, generator=g, device=cuda_device).to(bf)
                w = (torch.randn(h, generator=g, device=cuda_device) * 0.1 + 1).to(bf)
                assert lib.ako_b200_rmsnorm_set_staging(mode, 1 if mode == 2 else 0, 1 if mode == 2 else 0) == 0
                assert lib.ako_b200_measure_set_wait_polls(0) == 1 << 24
                if fused:
                    y, ro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
                else:
                    y = kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
                lib.ako_b200_measure_set_wait_polls(1 << 24)
                torch.cuda.synchronize()
                assert torch.isnan(y.float()).all(), (mode, h)
                if fused:
                    assert torch.isnan(ro.float()).all()
                # every entry point of this library now refuses, before launching
                with pytest.raises(RuntimeError, match="bounded wait"):
                    kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
                with pytest.raises(RuntimeError, match="bounded wait"):
                    kernels.swiglu_cuda_sm100(x, x)
                assert _native.take_device_status() == 1
                assert _native.take_device_status() == 0
                # accepted again, and correct
                lib.ako_b200_rmsnorm_set_staging(mode, 1 if mode == 2 else 0, 1 if mode == 2 else 0)
                y = kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
                check_rmsnorm(to_numpy(x[:3]), None, to_numpy(w), 1e-6, O.BF16, to_numpy(y[:3]), what="after expiry")
        finally:
            lib.ako_b200_measure_set_wait_polls(1 << 24)
            lib.ako_b200_rmsnorm_set_staging(0, 0, 0)
    # the product library never saw an expiry
    assert _native.take_device_status() == 0
    x = torch.randn(8, 4096, device=cuda_device).to(bf)
    assert torch.isfinite(kernels.rmsnorm_cuda_sm100(x, torch.ones(4096, device=cuda_device, dtype=bf)).float()).all()


def _kernel_names(fn) -> str:
    """Names of the CUDA kernels ``fn`` launches, from torch's profiler."""
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA], acc_events=True) as prof:
        fn()
        torch.cuda.synchronize()
    return " ".join(e.name for e in prof.events())


def test_launch_plan_matches_the_launched_kernel(cuda_device) -> None:
    """``ako_b200_rmsnorm_plan`` (host only) names the kernel and launch shape
    that the call then runs: the profiler's kernel name carries the same
    kernel and, for the row-resident kernel, the same template shape."""
    import ctypes
    import re

    lib = _native.lib()
    names = {0: "rms_rows_kernel", 1: "rms_tma_kernel", 2: "rms_chunk_kernel", 3: "rms_generic_kernel"}
    codes = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
    cases = [(32768, 16384, torch.bfloat16, True), (2048, 4096, torch.float32, False), (8192, 5120, torch.bfloat16, True),
             (8192, 5120, torch.float16, False), (32768, 1024, torch.bfloat16, False), (1, 16384, torch.bfloat16, True),
             (8192, 32768, torch.bfloat16, False), (2048, 65536, torch.float16, False), (4096, 65536, torch.bfloat16, True),
             (8192, 4100, torch.bfloat16, False), (16384, 1536, torch.float32, False)]
    for rows, h, dt, residual in cases:
        out = [ctypes.c_int() for _ in range(4)]
        assert lib.ako_b200_rmsnorm_plan(rows, h, codes[dt], int(residual), 1, *(ctypes.byref(o) for o in out)) == 0
        kernel, cluster, tpr, nv = (o.value for o in out)
        x = torch.randn(rows, h, device=cuda_device).to(dt)
        w = torch.ones(h, device=cuda_device, dtype=dt)
        if residual:
            got = _kernel_names(lambda: kernels.rmsnorm_residual_cuda_sm100(x, x, w, 1e-5))
        else:
            got = _kernel_names(lambda: kernels.rmsnorm_cuda_sm100(x, w, 1e-6))
        assert names[kernel] in got, (rows, h, dt, residual, kernel, got[:200])
        if kernel == 0:
            m = re.search(r"rms_rows_kernel<[^,]+, (\d+), (\d+), (?:true|false|1|0), (\d+)>", got)
            assert m is not None, got[:300]
            assert (int(m.group(3)), int(m.group(1)), int(m.group(2))) == (cluster, tpr, nv), (rows, h, got[:300])
        del x

    # SwiGLU: swiglu_kernel<T, VEC, UNROLL, FLAT, NARROW, THREADS, NC>
    for rows, f, dt, packed in ((16384, 14336, torch.bfloat16, False), (16384, 14336, torch.bfloat16, True),
                                (64, 14336, torch.float16, False), (1, 14336, torch.float16, False),
                                (7, 100, torch.bfloat16, False)):
        out = [ctypes.c_int() for _ in range(4)]
        assert lib.ako_b200_swiglu_plan(rows, f, codes[dt], 1, int(not packed), *(ctypes.byref(o) for o in out)) == 0
        access, threads, unroll, _ = (o.value for o in out)
        both = torch.randn(rows, 2 * f, device=cuda_device).to(dt)
        g, u = (both[:, :f], both[:, f:]) if packed else (both[:, :f].contiguous(), both[:, f:].contiguous())
        got = _kernel_names(lambda: kernels.swiglu_cuda_sm100(g, u))
        m = re.search(r"swiglu_kernel<[^,]+, (\d+), (\d+), (?:true|false|1|0), (?:true|false|1|0), (\d+)"
                      r"(?:, (?:true|false|1|0))?>", got)
        assert m is not None, got[:300]
        es = torch.tensor([], dtype=dt).element_size()
        assert (int(m.group(1)) * es, int(m.group(3)), int(m.group(2))) == (access, threads, unroll), (rows, f, got[:300])

    # RoPE: rope_vec_kernel<T, NP, INTERLEAVED, HPT>, or the pair-per-thread kernel
    for b, sq, hh, d, style in ((32, 512, 32, 128, "neox"), (8, 1, 8, 128, "neox"), (1, 1, 32, 128, "neox"),
                                (8, 64, 32, 128, "interleaved"), (8, 64, 8, 98, "neox")):
        out = [ctypes.c_int() for _ in range(5)]
        assert lib.ako_b200_rope_plan(b, sq, hh, d, 0 if style == "neox" else 1, 2, *(ctypes.byref(o) for o in out)) == 0
        access, hpt = out[0].value, out[1].value
        x = torch.randn(b, sq, hh, d, device=cuda_device).to(torch.bfloat16)
        cos, sin = (to_torch(t, O.F32, cuda_device) for t in O.build_rope_tables(sq, d))
        got = _kernel_names(lambda: kernels.rope_cuda_sm100(x, cos, sin, style))
        if d % 4 == 0:
            m = re.search(r"rope_vec_kernel<[^,]+, (\d+), (?:true|false|1|0), (\d+)>", got)
            assert m is not None, got[:300]
            assert (int(m.group(1)) * 2, int(m.group(2))) == (access, hpt), (b, sq, hh, d, style, got[:300])
        else:
            assert "rope_scalar_kernel" in got and access == 2, got[:300]


@pytest.mark.parametrize("dtype", DTYPES)
def test_wide_rows_staged_kernel(cuda_device, dtype: str) -> None:
    """Rows of 2049-8192 vectors through the 1024-thread staged kernel (the
    built-in choice for plain 16-bit rows of 16385-32768 elements from 1024
    rows on; forced for fp32, fused and 65536-wide rows) and through the
    chunked kernel (plain rows of 4097-8192 vectors, full and partial second
    chunks). Both keep the row-resident kernel's thread layout (1024 threads
    x 4 or 8 vectors) and sums, so the outputs are bit-identical to it; rows
    are checked against the oracle; uneven rows per CTA, a strided view, and
    no bounded wait ran out. Forced kernels run through the measurement build."""
    with _native.measurement() as lib:
        _wide_rows_cases(lib, cuda_device, dtype)


def _wide_rows_cases(lib, cuda_device, dtype: str) -> None:
    es = 4 if dtype == O.F32 else 2
    tdt = TORCH_DTYPE[dtype]
    g = torch.Generator(device=cuda_device).manual_seed(7)

    def rand(shape, mean=0.0, std=1.0):
        return (torch.randn(shape, generator=g, device=cuda_device) * std + mean).to(tdt)

    wide = 65536 // (es // 2) if es != 4 else 32768  # 8192 vectors
    cases = [(2048, 16392, 0), (2051, 24576, 0), (2048, 32768, 0), (300, 32768, 2), (257, wide, 2),
             (257, wide, 3), (300, wide - 8 // (es // 2) if es == 2 else wide - 4, 3), (150, 40968 // (es // 2), 3),
             (512, wide, 0)]
    if es == 2:  # one chunk per row: the row-resident kernel has the same 1024 x 4 layout
        cases += [(300, 32768, 3), (257, 24584, 3), (2049, 16392, 3)]
    try:
        for rows, h, mode in cases:
            x, r, w = rand((rows, h)), rand((rows, h)), rand((h,), 1.0, 0.1)
            forced = 1 if mode == 2 else 0  # one stage, one CTA per SM: the ring holds one wide row
            assert lib.ako_b200_rmsnorm_set_staging(mode, forced, forced) == 0
            y = kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
            expect = {2: "rms_tma_kernel", 3: "rms_chunk_kernel"}.get(mode)
            if mode == 0 and es == 2 and 16384 < h <= 32768 and rows >= 1024:
                expect = "rms_tma_kernel"
            if mode == 0 and es == 2 and h > 32768 and rows >= (128 if dtype == O.F16 else 1024):
                expect = "rms_chunk_kernel"
            if expect:
                assert expect in _kernel_names(lambda: kernels.rmsnorm_cuda_sm100(x, w, 1e-6)), (dtype, rows, h, mode)
            fused = h * es <= 65536  # two rows of the ring fit its 200 KB
            if fused:
                yr, ro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
            assert lib.ako_b200_rmsnorm_set_staging(1, 0, 0) == 0
            assert torch.equal(y, kernels.rmsnorm_cuda_sm100(x, w, 1e-6)), (dtype, rows, h, mode)
            if fused:
                yr1, ro1 = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
                assert torch.equal(ro, ro1) and torch.equal(yr, yr1), (dtype, rows, h, mode)
            sel = [0, 1, rows // 2, rows - 1]
            xs, wn = to_numpy(x[sel]), to_numpy(w)
            check_rmsnorm(xs, None, wn, 1e-6, dtype, to_numpy(y[sel]), what=f"wide h={h}")
            if fused:
                check_rmsnorm(xs, to_numpy(r[sel]), wn, 1e-5, dtype, to_numpy(yr[sel]), to_numpy(ro[sel]),
                              what=f"wide h={h}")
        # a strided view through the built-in choice
        assert lib.ako_b200_rmsnorm_set_staging(0, 0, 0) == 0
        base = rand((2048, 32768 + 64))
        xv, w = base[:, 64:], rand((32768,), 1.0, 0.1)
        y = kernels.rmsnorm_cuda_sm100(xv, w, 1e-6)
        assert_parity(C.rmsnorm(to_numpy(xv[:8]), to_numpy(w), 1e-6, dtype), to_numpy(y[:8]), dtype, "rmsnorm",
                      "wide strided")
        # both persistent kernels captured in a CUDA graph replay the eager bytes
        for rows, h in ((1024, 32768), (1024, 65536 // (es // 2) if es == 2 else 32768)):
            xg, wg = rand((rows, h)), rand((h,), 1.0, 0.1)
            mode = 0 if es == 2 else 2
            assert lib.ako_b200_rmsnorm_set_staging(mode, 1 if mode == 2 else 0, 1 if mode == 2 else 0) == 0
            eager = kernels.rmsnorm_cuda_sm100(xg, wg, 1e-6)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                kernels.rmsnorm_cuda_sm100(xg, wg, 1e-6)
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                yg = kernels.rmsnorm_cuda_sm100(xg, wg, 1e-6)
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(yg, eager), (dtype, rows, h)
            del graph
        torch.cuda.synchronize()
        assert _native.take_device_status() == 0
    finally:
        lib.ako_b200_rmsnorm_set_staging(0, 0, 0)


def test_rmsnorm_leading_dims_and_empty(cuda_device) -> None:
    rng = np.random.default_rng(9)
    x = normal(rng, (2, 3, 5, 512), 0, 1, O.BF16)
    w = normal(rng, (512,), 1, 0.1, O.BF16)
    y = kernels.rmsnorm_cuda_sm100(to_torch(x, O.BF16, cuda_device), to_torch(w, O.BF16, cuda_device))
    assert y.shape == (2, 3, 5, 512)
    assert_parity(C.rmsnorm(x, w, 1e-6, O.BF16), to_numpy(y), O.BF16, "rmsnorm", "4-d")
    empty = torch.empty(0, 512, dtype=torch.bfloat16, device=cuda_device)
    assert kernels.rmsnorm_cuda_sm100(empty, to_torch(w, O.BF16, cuda_device)).shape == (0, 512)


def test_offsets_beyond_2_31_elements(cuda_device) -> None:
    """Tensors of more than 2^31 elements (4.3 GB in bf16): every op's last
    rows sit past any 32-bit element offset. Their outputs, and the first
    rows', match the oracle (a wrapped offset would write the wrong rows)."""
    g = torch.Generator(device=cuda_device).manual_seed(3)
    bf = torch.bfloat16

    def rand(*shape):
        return torch.randn(*shape, generator=g, device=cuda_device).to(bf)

    def ends(t):
        return torch.cat([t[:2], t[-3:]])

    h = 4096
    rows = (1 << 31) // h + 3
    x, r, w = rand(rows, h), rand(rows, h), rand(h)
    y, ro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
    y_ref, ro_ref = C.rmsnorm_residual(to_numpy(ends(x)), to_numpy(ends(r)), to_numpy(w), 1e-5, O.BF16)
    np.testing.assert_array_equal(to_numpy(ends(ro)), ro_ref)
    assert_parity(y_ref, to_numpy(ends(y)), O.BF16, "rmsnorm_residual", "beyond 2^31")
    del r, ro, y
    y = kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
    assert_parity(C.rmsnorm(to_numpy(ends(x)), to_numpy(w), 1e-6, O.BF16), to_numpy(ends(y)), O.BF16, "rmsnorm",
                  "beyond 2^31")
    del x, y

    f = 14336
    m = (1 << 31) // f + 3
    gate, up = rand(m, f) * 2, rand(m, f) * 2
    y = kernels.swiglu_cuda_sm100(gate, up)
    assert_parity(C.swiglu(to_numpy(ends(gate)), to_numpy(ends(up)), O.BF16), to_numpy(ends(y)), O.BF16, "swiglu",
                  "beyond 2^31")
    del gate, up, y

    s = (1 << 31) // (32 * 128) + 2
    q = rand(1, s, 32, 128)
    cos, sin = (torch.from_numpy(t).to(cuda_device) for t in O.build_rope_tables(s, 128))
    y = kernels.rope_cuda_sm100(q, cos, sin, "neox")
    for lo, hi in ((0, 2), (s - 2, s)):
        ref = C.rope(to_numpy(q[:, lo:hi]), to_numpy(cos[lo:hi]), to_numpy(sin[lo:hi]), "neox", O.BF16)
        np.testing.assert_array_equal(to_numpy(y[:, lo:hi]), ref)


def test_rmsnorm_rejects_oversized_hidden_dim(cuda_device) -> None:
    x = torch.randn(1, kernels.MAX_HIDDEN_DIM + 2, device=cuda_device)
    with pytest.raises(ValueError, match="hidden_dim"):
        kernels.rmsnorm_residual_cuda_sm100(x, x, torch.ones(kernels.MAX_HIDDEN_DIM + 2, device=cuda_device))


# -------------------------------------------------------------------- rope
ROPE_SHAPES = [(2, 6, 3, 8), (1, 1, 32, 128), (8, 1, 8, 128), (32, 1, 8, 128), (2, 128, 8, 64), (1, 64, 32, 128),
               (3, 17, 5, 128), (2, 9, 4, 256), (1, 5, 2, 6), (2, 4, 3, 2),
               # half head sizes that take 8-byte (36 pairs) and 4-byte (50, 10 pairs) accesses
               (2, 9, 3, 100), (1, 7, 4, 72), (2, 5, 6, 20)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("style", O.ROPE_STYLES)
@pytest.mark.parametrize("shape", ROPE_SHAPES, ids=[str(s) for s in ROPE_SHAPES])
def test_rope_shapes(cuda_device, dtype: str, style: str, shape) -> None:
    b, s, h, d = shape
    rng = np.random.default_rng(b * 1000 + s * 10 + h)
    x = normal(rng, shape, 0, 1, dtype)
    cos, sin = O.build_rope_tables(s, d, offset=3)
    y = kernels.rope_cuda_sm100(to_torch(x, dtype, cuda_device), to_torch(cos, O.F32, cuda_device),
                                to_torch(sin, O.F32, cuda_device), style)
    np.testing.assert_array_equal(to_numpy(y), O.rope(x, cos, sin, style, dtype))


@pytest.mark.parametrize("style", O.ROPE_STYLES)
@pytest.mark.parametrize("dtype", DTYPES)
def test_rope_views_at_every_alignment(cuda_device, dtype: str, style: str) -> None:
    """Views starting 0..3 elements into a padded buffer: each start selects a
    different access width (16, 8, 4 bytes or element accesses)."""
    rng = np.random.default_rng(31)
    b, s, hh, d = 2, 9, 5, 128
    cos, sin = O.build_rope_tables(s, d, offset=7)
    base = to_torch(normal(rng, (b, s, hh, d + 8), 0, 1, dtype), dtype, cuda_device)
    for off in range(4):
        x = base[..., off:off + d]
        y = kernels.rope_cuda_sm100(x, to_torch(cos, O.F32, cuda_device), to_torch(sin, O.F32, cuda_device), style)
        np.testing.assert_array_equal(to_numpy(y), O.rope(to_numpy(x), cos, sin, style, dtype), err_msg=f"offset {off}")


@pytest.mark.parametrize("style", O.ROPE_STYLES)
@pytest.mark.parametrize("dtype", (O.F16, O.BF16))
def test_rope_bhsd_transposed_view_and_table_slice(cuda_device, dtype: str, style: str) -> None:
    """q stored (B, H, S, D) and passed as .transpose(1, 2); decode-style
    table slice cos[2047:2048] of an 8192-row table; neither is copied."""
    rng = np.random.default_rng(21)
    cos_full, sin_full = O.build_rope_tables(8192, 128)
    cos_d, sin_d = to_torch(cos_full, O.F32, cuda_device), to_torch(sin_full, O.F32, cuda_device)
    for b, hh, s, off in ((4, 32, 1, 2047), (2, 8, 33, 100)):
        q_bhsd = normal(rng, (b, hh, s, 128), 0, 1, dtype)
        q = to_torch(q_bhsd, dtype, cuda_device).transpose(1, 2)
        y = kernels.rope_cuda_sm100(q, cos_d[off:off + s], sin_d[off:off + s], style)
        assert y.stride() == q.stride()  # the output keeps the (B, H, S, D) layout
        ref = O.rope(np.ascontiguousarray(q_bhsd.transpose(0, 2, 1, 3)), cos_full[off:off + s],
                     sin_full[off:off + s], style, dtype)
        np.testing.assert_array_equal(to_numpy(y), ref)


@pytest.mark.parametrize("hpt", [1, 2, 4])
@pytest.mark.parametrize("style", O.ROPE_STYLES)
def test_rope_every_heads_per_thread(cuda_device, hpt: int, style: str) -> None:
    """Each built heads-per-thread variant (forced through the measurement
    build), head counts not divisible by it."""
    rng = np.random.default_rng(hpt)
    with _native.measurement() as lib:
        try:
            assert lib.ako_b200_rope_set_launch(hpt) == 0
            for dtype in DTYPES:
                for b, s, hh, d in ((2, 7, 1, 128), (1, 3, 3, 64), (3, 5, 40, 128), (1, 9, 32, 128), (2, 2, 5, 16)):
                    x = normal(rng, (b, s, hh, d), 0, 1, dtype)
                    cos, sin = O.build_rope_tables(s, d, offset=11)
                    y = kernels.rope_cuda_sm100(to_torch(x, dtype, cuda_device), to_torch(cos, O.F32, cuda_device),
                                                to_torch(sin, O.F32, cuda_device), style)
                    np.testing.assert_array_equal(to_numpy(y), O.rope(x, cos, sin, style, dtype))
        finally:
            lib.ako_b200_rope_set_launch(0)


def test_rope_many_positions(cuda_device) -> None:
    """batch * seq well past 2^16 positions exercises the position split."""
    rng = np.random.default_rng(17)
    b, s, hh, d = 37, 4099, 2, 32
    x = normal(rng, (b, s, hh, d), 0, 1, O.BF16)
    cos, sin = O.build_rope_tables(s, d)
    y = kernels.rope_cuda_sm100(to_torch(x, O.BF16, cuda_device), to_torch(cos, O.F32, cuda_device),
                                to_torch(sin, O.F32, cuda_device), "neox")
    np.testing.assert_array_equal(to_numpy(y), C.rope(x, cos, sin, "neox", O.BF16))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("style", O.ROPE_STYLES)
def test_rope_qk_fused_matches_two_ropes(cuda_device, dtype: str, style: str) -> None:
    """One launch for q (32 heads) and k (8 heads) equals two rope calls and the
    oracle, bit for bit; q passed as a (B, H, S, D) transposed view, k dense,
    decode-style table slice."""
    rng = np.random.default_rng(23)
    cos_full, sin_full = O.build_rope_tables(8192, 128)
    for b, s, off in ((4, 1, 2047), (2, 33, 0), (1, 5, 100)):
        q_np = normal(rng, (b, 32, s, 128), 0, 1, dtype)  # (B, H, S, D) storage
        k_np = normal(rng, (b, s, 8, 128), 0, 1, dtype)
        q = to_torch(q_np, dtype, cuda_device).transpose(1, 2)
        k = to_torch(k_np, dtype, cuda_device)
        cos = to_torch(cos_full, O.F32, cuda_device)[off:off + s]
        sin = to_torch(sin_full, O.F32, cuda_device)[off:off + s]
        qo, ko = kernels.rope_qk_cuda_sm100(q, k, cos, sin, style)
        assert qo.stride() == q.stride()
        assert torch.equal(qo, kernels.rope_cuda_sm100(q, cos, sin, style))
        assert torch.equal(ko, kernels.rope_cuda_sm100(k, cos, sin, style))
        ref_q = O.rope(np.ascontiguousarray(q_np.transpose(0, 2, 1, 3)), cos_full[off:off + s],
                       sin_full[off:off + s], style, dtype)
        np.testing.assert_array_equal(to_numpy(qo), ref_q)
        np.testing.assert_array_equal(to_numpy(ko), O.rope(k_np, cos_full[off:off + s], sin_full[off:off + s],
                                                           style, dtype))


def test_rope_qk_validation(cuda_device) -> None:
    q = torch.randn(2, 4, 8, 64, device=cuda_device, dtype=torch.bfloat16)
    cos = torch.ones(4, 32, device=cuda_device)
    with pytest.raises(ValueError):
        kernels.rope_qk_cuda_sm100(q, q[:, :3], cos, cos)
    with pytest.raises(ValueError):
        kernels.rope_qk_cuda_sm100(q, q.float(), cos, cos)
    qo, ko = kernels.rope_qk_cuda_sm100(q, q[:, :, :0], cos, torch.zeros_like(cos))
    assert torch.equal(qo, q) and ko.shape == (2, 4, 0, 64)


def test_rope_position_zero_identity_and_empty(cuda_device) -> None:
    x = torch.randn(2, 3, 4, 64, device=cuda_device, dtype=torch.bfloat16)
    cos = torch.ones(3, 32, device=cuda_device)
    sin = torch.zeros(3, 32, device=cuda_device)
    assert torch.equal(kernels.rope_cuda_sm100(x, cos, sin), x)
    e = torch.empty(0, 3, 4, 64, device=cuda_device, dtype=torch.bfloat16)
    assert kernels.rope_cuda_sm100(e, cos, sin).shape == e.shape


# ------------------------------------------------------------------ swiglu
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(1, 5632), (64, 11008), (7, 100), (3, 14336), (2, 3, 8448), (1, 1), (33, 24),
                                   (2, 11008), (2, 16384), (1, 32776)])
def test_swiglu_shapes(cuda_device, dtype: str, shape) -> None:
    rng = np.random.default_rng(sum(shape))
    g = normal(rng, shape, 0, 2, dtype)
    u = normal(rng, shape, 0, 2, dtype)
    y = kernels.swiglu_cuda_sm100(to_torch(g, dtype, cuda_device), to_torch(u, dtype, cuda_device))
    assert y.shape == g.shape
    assert_parity(C.swiglu(g, u, dtype), to_numpy(y), dtype, "swiglu", f"swiglu {shape}")


@pytest.mark.parametrize("dtype", DTYPES)
def test_swiglu_packed_halves(cuda_device, dtype: str) -> None:
    """One [M, 2F] projection output split into gate and up views, no copy."""
    rng = np.random.default_rng(13)
    for m, f in ((64, 5632), (1, 11008), (5, 100)):
        packed = normal(rng, (m, 2 * f), 0, 2, dtype)
        p = to_torch(packed, dtype, cuda_device)
        y = kernels.swiglu_cuda_sm100(p[:, :f], p[:, f:])
        ref = C.swiglu(np.ascontiguousarray(packed[:, :f]), np.ascontiguousarray(packed[:, f:]), dtype)
        assert_parity(ref, to_numpy(y), dtype, "swiglu", f"packed {m}x{f}")


@pytest.mark.parametrize("dtype", (O.F16, O.BF16))
def test_swiglu_every_16bit_pattern(cuda_device, dtype: str) -> None:
    """Every finite 16-bit pattern as the gate and as the up input (the other
    operand kept where the product stays finite), against the oracle: covers
    the kernel's conversions of subnormals, signed zeros and the largest
    values; infinities and NaN give the oracle's classes."""
    rng = np.random.default_rng(17)
    bits = np.arange(65536, dtype=np.uint16)
    exp_mask = 0x7C00 if dtype == O.F16 else 0x7F80
    finite = bits[(bits & exp_mask) != exp_mask]
    vals = finite.view(np.float16) if dtype == O.F16 else finite

    def enc(a: np.ndarray) -> np.ndarray:
        return O.encode(a.astype(np.float32), dtype) if dtype == O.BF16 else a.astype(np.float16)

    n = vals.size
    for g, u in ((vals, enc(rng.uniform(-0.9, 0.9, n))), (enc(rng.uniform(-1.0, 0.5, n)), vals)):
        g2, u2 = g.reshape(1, n), u.reshape(1, n)
        y = kernels.swiglu_cuda_sm100(to_torch(g2, dtype, cuda_device), to_torch(u2, dtype, cuda_device))
        assert_parity(C.swiglu(g2, u2, dtype), to_numpy(y), dtype, "swiglu", "every pattern")
    special = np.array([[np.inf, -np.inf, np.nan, 1.0, -1.0, 0.0, np.nan, 2.0]], dtype=np.float32)
    ones = np.array([[1.0, 1.0, 1.0, np.inf, np.inf, np.inf, 1.0, np.nan]], dtype=np.float32)
    gs, us = enc(special), enc(ones)
    y = kernels.swiglu_cuda_sm100(to_torch(gs, dtype, cuda_device), to_torch(us, dtype, cuda_device))
    ref = O.decode(C.swiglu(gs, us, dtype), dtype)
    out = O.decode(to_numpy(y), dtype)
    np.testing.assert_array_equal(np.isnan(out), np.isnan(ref))
    np.testing.assert_array_equal(out[~np.isnan(ref)], ref[~np.isnan(ref)])


def test_swiglu_extremes(cuda_device) -> None:
    g = torch.tensor([[-100.0, -20.0, -1.0, 0.0, 1.0, 20.0, 100.0, float("inf")]], device=cuda_device)
    u = torch.ones_like(g)
    y = kernels.swiglu_cuda_sm100(g, u).cpu()
    ref = C.swiglu(to_numpy(g), to_numpy(u), O.F32)
    # expf of large arguments may differ by an ulp between CUDA and libm.
    np.testing.assert_allclose(y.numpy()[:, :7], ref[:, :7], rtol=4 * 2.0**-23, atol=0)
    assert torch.isinf(y[0, 7])


# ------------------------------------------------------- launch semantics
def test_programmatic_launch_changes_no_result(cuda_device) -> None:
    """Every kernel runs with and without programmatic dependent launch; chains
    of dependent calls (each reads the previous call's output) give identical
    bytes both ways, eagerly and in a CUDA graph (the switch exists in the
    measurement build; the product library always launches programmatically
    and gives the same bytes)."""
    cos, sin = (to_torch(t, O.F32, cuda_device) for t in O.build_rope_tables(96, 128))
    x = torch.randn(96, 4096, device=cuda_device, dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.randn(4096, device=cuda_device, dtype=torch.bfloat16)

    def chain():
        y, ro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
        y2 = kernels.rmsnorm_cuda_sm100(ro, w, 1e-6)
        q = kernels.rope_cuda_sm100(y2.view(1, 96, 32, 128), cos[:96], sin[:96], "neox")
        return kernels.swiglu_cuda_sm100(q.view(96, 4096), y)

    def run() -> tuple[torch.Tensor, torch.Tensor]:
        eager = chain()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            chain()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            captured = chain()
        graph.replay()
        torch.cuda.synchronize()
        out = (eager.clone(), captured.clone())
        del graph
        return out

    outs = {"product": run()}
    with _native.measurement() as lib:
        try:
            for pdl in (0, 1):
                lib.ako_b200_set_pdl(pdl)
                outs[pdl] = run()
        finally:
            lib.ako_b200_set_pdl(1)
    ref = outs[0][0]
    for eager, captured in outs.values():
        assert torch.equal(eager, ref) and torch.equal(captured, ref)


@pytest.mark.parametrize("dtype", (O.BF16, O.F32))
def test_host_buffer_pipeline_matches_the_device_call(cuda_device, dtype: str) -> None:
    """The host-buffer entry point (pinned host tensors streamed through the
    GPU in chunks on three streams), for several chunk and slot counts with a
    ragged last chunk: the rounded residual equals the device call's bytes;
    the norm is within the parity gates (a chunk's row count can select
    another launch shape, whose reduction order differs) and equals the
    device call's bytes when one chunk holds every row."""
    from ako_b200 import host

    rng = np.random.default_rng(41)
    rows, h = 1000, 4096
    x, r = normal(rng, (rows, h), 0, 1, dtype), normal(rng, (rows, h), 0, 1, dtype)
    w = normal(rng, (h,), 1, 0.1, dtype)
    wd = to_torch(w, dtype, cuda_device)
    yd, rod = kernels.rmsnorm_residual_cuda_sm100(to_torch(x, dtype, cuda_device), to_torch(r, dtype, cuda_device),
                                                  wd, 1e-5)
    xh, rh = to_torch(x, dtype, "cpu").pin_memory(), to_torch(r, dtype, "cpu").pin_memory()
    y_ref, ro_ref = C.rmsnorm_residual(x, r, w, 1e-5, dtype)
    for chunk_rows, slots in ((96, 3), (333, 2), (1000, 3), (7, 4)):
        y, ro = host.rmsnorm_residual_host(xh, rh, wd, 1e-5, chunk_rows=chunk_rows, slots=slots)
        torch.cuda.current_stream().synchronize()
        what = f"chunks of {chunk_rows}, {slots} slots"
        assert torch.equal(ro, rod.cpu()), what
        np.testing.assert_array_equal(to_numpy(ro), ro_ref)
        assert_parity(y_ref, to_numpy(y), dtype, "rmsnorm_residual", what)
        if chunk_rows >= rows:
            assert torch.equal(y, yd.cpu()), what
    # preallocated pinned outputs are filled in place
    y_out = torch.empty_like(xh).pin_memory()
    ro_out = torch.empty_like(xh).pin_memory()
    host.rmsnorm_residual_host(xh, rh, wd, 1e-5, y_out=y_out, residual_out=ro_out, chunk_rows=rows)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(y_out, yd.cpu()) and torch.equal(ro_out, rod.cpu())
    with pytest.raises(ValueError, match="host tensors"):
        host.rmsnorm_residual_host(xh.to(cuda_device), rh, wd)
    with pytest.raises(ValueError, match="weight must live"):
        host.rmsnorm_residual_host(xh, rh, wd.cpu())


def test_runs_on_the_current_stream_and_in_a_graph(cuda_device) -> None:
    x = torch.randn(64, 4096, device=cuda_device, dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.randn(4096, device=cuda_device, dtype=torch.bfloat16)
    eager_y, eager_ro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gy, gro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
        gs = kernels.swiglu_cuda_sm100(x, r)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gy, eager_y) and torch.equal(gro, eager_ro)
    assert torch.equal(gs, kernels.swiglu_cuda_sm100(x, r))


def test_wrong_device_and_dtype_errors(cuda_device) -> None:
    x = torch.randn(2, 64, device=cuda_device, dtype=torch.float64)
    with pytest.raises(ValueError, match="float32/float16/bfloat16"):
        kernels.rmsnorm_cuda_sm100(x, torch.ones(64, device=cuda_device, dtype=torch.float64))
    with pytest.raises(ValueError, match="weight"):
        kernels.rmsnorm_cuda_sm100(x.float(), torch.ones(64))


# ------------------------------------------------- full benchmark sizes
def test_full_size_residual_against_torch_fp32(cuda_device) -> None:
    """Config 2's largest cell (32768 x 16384 bf16): the rounded residual is
    exact against torch's own add; the norm is within budget of an fp32 torch
    evaluation of the reference formula; 64 sampled rows match the oracle."""
    torch.manual_seed(0)
    m, h = 32768, 16384
    x = torch.randn(m, h, device=cuda_device, dtype=torch.bfloat16)
    r = torch.randn(m, h, device=cuda_device, dtype=torch.bfloat16)
    w = (torch.randn(h, device=cuda_device) * 0.1 + 1).to(torch.bfloat16)
    y, ro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
    assert torch.equal(ro, x + r)
    for lo in range(0, m, 4096):  # the fp32 reference in slabs bounds the extra memory
        rs = ro[lo:lo + 4096].float()
        ref = (rs * torch.rsqrt(rs.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()).to(torch.bfloat16)
        diff = (ref.float() - y[lo:lo + 4096].float()).abs().max().item()
        assert diff <= 1e-5 + 1.6e-2 * ref.float().abs().max().item()
    idx = torch.randint(0, m, (64,), device=cuda_device)
    xs, rs_ = to_numpy(x[idx]), to_numpy(r[idx])
    y_ref, ro_ref = C.rmsnorm_residual(xs, rs_, to_numpy(w), 1e-5, O.BF16)
    np.testing.assert_array_equal(to_numpy(ro[idx]), ro_ref)
    assert_parity(y_ref, to_numpy(y[idx]), O.BF16, "rmsnorm_residual", "full-size sample")


def test_full_size_rope_and_swiglu_properties(cuda_device) -> None:
    """Config 3's largest q (32 x 4096 x 32 x 128) and config 4's largest
    swiglu (16384 x 14336), bf16: RoPE matches torch's fp32 evaluation of the
    reference expression bit for bit; SwiGLU is within budget of torch's fp32
    silu(g) * u, and zero wherever up is zero."""
    torch.manual_seed(1)
    b, s, hh, d = 32, 4096, 32, 128
    q = torch.randn(b, s, hh, d, device=cuda_device, dtype=torch.bfloat16)
    cos_np, sin_np = O.build_rope_tables(s, d)
    cos, sin = to_torch(cos_np, O.F32, cuda_device), to_torch(sin_np, O.F32, cuda_device)
    y = kernels.rope_cuda_sm100(q, cos, sin, "neox")
    for lo in range(0, b, 4):
        qc = q[lo:lo + 4].float()
        x0, x1 = qc[..., :64], qc[..., 64:]
        c, sn = cos[None, :, None, :], sin[None, :, None, :]
        ref = torch.cat([x0 * c - x1 * sn, x0 * sn + x1 * c], dim=-1).to(torch.bfloat16)
        assert torch.equal(ref, y[lo:lo + 4])
    del q, y
    g = torch.randn(16384, 14336, device=cuda_device, dtype=torch.bfloat16) * 2
    u = torch.randn_like(g) * 2
    u[::7] = 0
    out = kernels.swiglu_cuda_sm100(g, u)
    assert not out[::7].float().abs().max().item()
    for lo in range(0, 16384, 2048):
        ref = (torch.nn.functional.silu(g[lo:lo + 2048].float()) * u[lo:lo + 2048].float()).to(torch.bfloat16)
        diff = (ref.float() - out[lo:lo + 2048].float()).abs().max().item()
        assert diff <= 1e-5 + 1.6e-2 * ref.float().abs().max().item()


# ------------------------------------------------------------- randomized
def _view(base: torch.Tensor, rows: int, width: int, stride: int, off: int) -> torch.Tensor:
    """rows x width view with row stride `stride`, starting `off` elements into the flat `base`."""
    return base[off:].as_strided((rows, width), (stride, 1))


def test_randomized_shapes_and_offsets_against_oracle(cuda_device) -> None:
    """Seeded random widths, row counts, dtypes, row paddings and view offsets
    (every access width and the scalar paths), all three ops against the
    oracle."""
    rng = np.random.default_rng(2026)
    for case in range(48):
        dtype = DTYPES[case % 3]
        tdt = TORCH_DTYPE[dtype]
        rows = int(rng.integers(1, 70))
        h = int(rng.choice([int(rng.integers(1, 300)), int(rng.integers(300, 9000)), 4096, 4100, 8192]))
        pad = int(rng.integers(0, 9))
        off = int(rng.integers(0, 9))
        what = f"case {case}: {dtype} rows={rows} h={h} pad={pad} off={off}"

        def padded(width: int, start: int) -> torch.Tensor:
            a = normal(rng, (rows * (width + pad) + 16,), 0, 1, dtype)  # room for any start <= 16
            return _view(to_torch(a, dtype, cuda_device), rows, width, width + pad, start)

        x = padded(h, off)
        r = padded(h, off)
        w = to_torch(normal(rng, (h,), 1, 0.1, dtype), dtype, cuda_device)
        xn, rn, wn = to_numpy(x), to_numpy(r), to_numpy(w)
        y, ro = kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5)
        y_ref, ro_ref = C.rmsnorm_residual(xn, rn, wn, 1e-5, dtype)
        np.testing.assert_array_equal(to_numpy(ro), ro_ref, err_msg=what)
        assert_parity(y_ref, to_numpy(y), dtype, "rmsnorm_residual", what)
        assert_parity(C.rmsnorm(xn, wn, 1e-6, dtype), to_numpy(kernels.rmsnorm_cuda_sm100(x, w, 1e-6)), dtype,
                      "rmsnorm", what)

        g, u = padded(h, off), padded(h, (off + 3) % 9)
        assert_parity(C.swiglu(to_numpy(g), to_numpy(u), dtype), to_numpy(kernels.swiglu_cuda_sm100(g, u)), dtype,
                      "swiglu", what)

        d = 2 * int(rng.integers(1, 80))
        heads, seq = int(rng.integers(1, 9)), int(rng.integers(1, 9))
        style = O.ROPE_STYLES[case % 2]
        qbase = to_torch(normal(rng, (seq * heads * (d + pad) + 16,), 0, 1, dtype), dtype, cuda_device)
        q = qbase[off:].as_strided((1, seq, heads, d), (seq * heads * (d + pad), heads * (d + pad), d + pad, 1))
        cos, sin = O.build_rope_tables(seq, d, offset=int(rng.integers(0, 100)))
        yq = kernels.rope_cuda_sm100(q, to_torch(cos, O.F32, cuda_device), to_torch(sin, O.F32, cuda_device), style)
        np.testing.assert_array_equal(to_numpy(yq), O.rope(to_numpy(q), cos, sin, style, dtype),
                                      err_msg=f"{what} rope d={d} heads={heads} seq={seq} {style}")


def test_host_pipeline_keeps_few_slot_sets(cuda_device) -> None:
    """Calls of varying row counts reuse power-of-two slot capacities, and at
    most MAX_SLOT_SETS slot sets stay allocated; every call's outputs equal
    the device call's."""
    from ako_b200 import host

    host._slot_cache.clear()
    w = torch.randn(512, device=cuda_device).to(torch.bfloat16)
    for rows in (1, 3, 5, 17, 100, 129, 300, 700, 1500, 3000, 33, 6):
        x = torch.randn(rows, 512).to(torch.bfloat16).pin_memory()
        r = torch.randn(rows, 512).to(torch.bfloat16).pin_memory()
        y, ro = host.rmsnorm_residual_host(x, r, w, 1e-5, chunk_rows=1024)
        torch.cuda.current_stream().synchronize()
        yd, rod = kernels.rmsnorm_residual_cuda_sm100(x.to(cuda_device), r.to(cuda_device), w, 1e-5)
        assert torch.equal(y, yd.cpu()) and torch.equal(ro, rod.cpu()), rows
        assert len(host._slot_cache) <= host.MAX_SLOT_SETS
    assert {k[1] for k in host._slot_cache} <= {1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024}
