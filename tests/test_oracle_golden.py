"""The oracle, pinned: both CPU restatements reproduce the reference's own
outputs (golden vectors made by ``tests/golden/make_golden.py`` from
``ako.ops.*_ref``) within the parity gates, and the known answers and
properties of the reference's tests hold for them."""

from __future__ import annotations

import numpy as np
import pytest

import golden_data as gd
from helpers import assert_parity, normal
from oracle import ako_oracle as O
from oracle import c_oracle as C

ALL = gd.cases()


def _run(impl, case):
    dt = case["dtype"]
    op = case["op"]
    a = lambda k: gd.arr(case, k)  # noqa: E731
    if op == "rmsnorm":
        return {"y": impl.rmsnorm(a("x"), a("w"), case["eps"], dt)}
    if op == "rmsnorm_residual":
        y, ro = impl.rmsnorm_residual(a("x"), a("r"), a("w"), case["eps"], dt)
        return {"y": y, "ro": ro}
    if op == "rope":
        return {"y": impl.rope(a("x"), a("cos"), a("sin"), case["style"], dt)}
    return {"y": impl.swiglu(a("g"), a("u"), dt)}


@pytest.mark.parametrize("impl", [O, C], ids=["numpy", "c"])
@pytest.mark.parametrize("case", ALL, ids=[c["name"] for c in ALL])
def test_oracle_matches_reference_golden(impl, case) -> None:
    out = _run(impl, case)
    dt = case["dtype"]
    if "ro" in out:  # the rounded residual is exact
        np.testing.assert_array_equal(out["ro"], gd.arr(case, "ro"))
    if case["op"] == "rope":  # separate products and a sum: bit-exact
        np.testing.assert_array_equal(out["y"], gd.arr(case, "y"))
    assert_parity(gd.arr(case, "y"), out["y"], dt, case["op"], case["name"])


def test_known_answer() -> None:
    """Reference tests/test_rmsnorm.py:24-29: [[3, 4]] -> x / sqrt(12.5)."""
    x = np.array([[3.0, 4.0]], np.float32)
    y = O.rmsnorm(x, np.ones(2, np.float32), 1e-6, O.F32)
    np.testing.assert_allclose(y, x / np.sqrt(12.5), rtol=1e-6)
    yc = C.rmsnorm(x, np.ones(2, np.float32), 1e-6, O.F32)
    np.testing.assert_array_equal(y, yc)


def test_rope_tables_match_reference_rows() -> None:
    """Table rows the reference built: exact-ish near 0, within the fp32 angle
    error (2 ulp of pos * inv_freq, which the two pow implementations differ
    by) at large positions."""
    rows, cos_ref, sin_ref = gd.table_rows()
    cos, sin = O.build_rope_tables(8192, 128)
    for i, r in enumerate(rows):
        bound = 1.2e-7 + float(r) * 2.0**-22
        assert np.abs(cos[r] - cos_ref[i]).max() <= bound
        assert np.abs(sin[r] - sin_ref[i]).max() <= bound
    assert np.array_equal(cos[0], np.ones(64, np.float32)) and not sin[0].any()
    assert cos[1, 0] == pytest.approx(np.cos(1.0), abs=1e-6)


def test_rope_offset_and_identity() -> None:
    cos_full, sin_full = O.build_rope_tables(8, 8)
    cos_off, sin_off = O.build_rope_tables(4, 8, offset=4)
    np.testing.assert_allclose(cos_off, cos_full[4:], atol=1e-6)
    np.testing.assert_allclose(sin_off, sin_full[4:], atol=1e-6)
    x = normal(np.random.default_rng(0), (1, 3, 1, 8), 0, 1, O.F32)
    y = O.rope(x, *O.build_rope_tables(3, 8), "neox", O.F32)
    np.testing.assert_array_equal(y[:, 0], x[:, 0])


@pytest.mark.parametrize("style", O.ROPE_STYLES)
def test_rope_preserves_pair_norm(style: str) -> None:
    x = normal(np.random.default_rng(1), (2, 12, 2, 16), 0, 1, O.F32)
    y = O.rope(x, *O.build_rope_tables(12, 16), style, O.F32)
    np.testing.assert_allclose(np.linalg.norm(y, axis=-1), np.linalg.norm(x, axis=-1), rtol=1e-5)


def test_swiglu_zero_up_is_zero() -> None:
    g = normal(np.random.default_rng(2), (3, 16), 0, 2, O.BF16)
    assert not O.decode(O.swiglu(g, np.zeros_like(g), O.BF16), O.BF16).any()  # -0.0 counts as zero


@pytest.mark.parametrize("dtype", O.DTYPES)
def test_numpy_and_c_oracles_agree(dtype: str) -> None:
    rng = np.random.default_rng(3)
    x = normal(rng, (64, 4096), 0, 1, dtype)
    r = normal(rng, (64, 4096), 0, 1, dtype)
    w = normal(rng, (4096,), 1, 0.1, dtype)
    y_np, ro_np = O.rmsnorm_residual(x, r, w, 1e-5, dtype)
    y_c, ro_c = C.rmsnorm_residual(x, r, w, 1e-5, dtype, threads=4)
    np.testing.assert_array_equal(ro_np, ro_c)
    assert_parity(y_np, y_c, dtype, "rmsnorm_residual", "oracles")
    q = normal(rng, (2, 16, 8, 128), 0, 1, dtype)
    cos, sin = O.build_rope_tables(16, 128)
    for style in O.ROPE_STYLES:
        np.testing.assert_array_equal(O.rope(q, cos, sin, style, dtype), C.rope(q, cos, sin, style, dtype, threads=3))
    g = normal(rng, (32, 1000), 0, 2, dtype)
    u = normal(rng, (32, 1000), 0, 2, dtype)
    assert_parity(O.swiglu(g, u, dtype), C.swiglu(g, u, dtype, threads=2), dtype, "swiglu", "oracles")


def test_bf16_encode_rounds_to_nearest_even() -> None:
    f = np.array([1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, -2.5, np.inf, 0.0], np.float32)
    b = O.encode(f, O.BF16)
    np.testing.assert_array_equal(O.decode(b, O.BF16), np.array([1.0, 1.0, 1.0 + 2**-6, -2.5, np.inf, 0.0], np.float32))
    assert np.isnan(O.decode(O.encode(np.array([np.nan], np.float32), O.BF16), O.BF16)).all()


def test_ulp_distance_counts_steps() -> None:
    a = O.encode(np.array([1.0, -1.0, 0.0], np.float32), O.BF16)
    b = a.copy()
    b[0] += 2
    b[1] += 1  # more negative by one step
    np.testing.assert_array_equal(O.ulp_distance(a, b, O.BF16), [2, 1, 0])


# ---------------------------------------------------- the kernels' sum order
def _fixed_order_sum_py(sq: np.ndarray, vec: int) -> np.float32:
    """The CUDA RMSNorm kernels' summation order, restated with fp32 scalars:
    each vector's squares pairwise (1, 2, 4 apart), each group of 32
    vectors by a fold (16, 8, 4, 2, 1 apart), then the groups by the same
    fold, zero-padded to a power of two."""
    f = np.float32
    nvec = sq.size // vec
    vsum = []
    for v in range(nvec):
        e = [f(t) for t in sq[v * vec:(v + 1) * vec]]
        st = 1
        while st < vec:
            for i in range(0, vec - st, 2 * st):
                e[i] = f(e[i] + e[i + st])
            st *= 2
        vsum.append(e[0])

    def fold(vals: list) -> np.float32:
        n = 1
        while n < len(vals):
            n *= 2
        vals = vals + [f(0)] * (n - len(vals))
        off = n // 2
        while off >= 1:
            for i in range(off):
                vals[i] = f(vals[i] + vals[i + off])
            off //= 2
        return vals[0]

    groups = [fold(vsum[g:g + 32] + [f(0)] * (32 - len(vsum[g:g + 32]))) for g in range(0, nvec, 32)]
    return fold(groups)


@pytest.mark.parametrize("dtype", (O.F32, O.F16, O.BF16))
@pytest.mark.parametrize("h", (8, 64, 256, 264, 1000, 2048, 5128))
def test_fixed_order_model_follows_its_definition(dtype: str, h: int) -> None:
    """The C model of the kernels' summation order (the reference the GPU tests
    hold the kernels to, bit for bit) equals a plain restatement of the
    documented order, and stays within the reference gate of the
    reference-order oracle."""
    vec = 4 if dtype == O.F32 else 8
    if h % vec:
        pytest.skip("not whole 16-byte vectors")
    rng = np.random.default_rng(h)
    x = O.encode(rng.standard_normal((3, h), dtype=np.float32), dtype)
    w = O.encode(rng.standard_normal(h, dtype=np.float32) * np.float32(0.1) + 1, dtype)
    y = C.rmsnorm_fixed_order(x, None, w, 1e-6, dtype)
    xf, wf = O.decode(x, dtype).astype(np.float32), O.decode(w, dtype).astype(np.float32)
    for row in range(3):
        v = xf[row]
        total = _fixed_order_sum_py((v * v).astype(np.float32), vec)
        inv = np.float32(1) / np.sqrt(np.float32(total / np.float32(h)) + np.float32(1e-6), dtype=np.float32)
        expect = O.encode(((v * inv).astype(np.float32) * wf).astype(np.float32), dtype)
        np.testing.assert_array_equal(y[row], expect)
    assert int(O.ulp_distance(C.rmsnorm(x, w, 1e-6, dtype), y, dtype).max()) <= (1 if dtype != O.F32 else 4)


def test_fixed_order_model_against_reference_golden() -> None:
    """On the reference's own RMSNorm outputs (golden vectors with rows of
    whole 16-byte vectors) the fixed order is within 1 ulp for 16-bit
    outputs and within the fp32 elementwise bound."""
    from helpers import ULP_F32

    checked = 0
    for case in gd.cases():
        if case["op"] not in ("rmsnorm", "rmsnorm_residual"):
            continue
        dt = case["dtype"]
        x = gd.arr(case, "x")
        h = x.shape[-1]
        if (h * (4 if dt == O.F32 else 2)) % 16:
            continue
        r = gd.arr(case, "r") if case["op"] == "rmsnorm_residual" else None
        out = C.rmsnorm_fixed_order(x.reshape(-1, h), None if r is None else r.reshape(-1, h),
                                    gd.arr(case, "w"), case["eps"], dt)
        y = (out if r is None else out[0]).reshape(gd.arr(case, "y").shape)
        bound = 1 if dt != O.F32 else ULP_F32[case["op"]]
        assert int(O.ulp_distance(gd.arr(case, "y"), y, dt).max()) <= bound, case["name"]
        checked += 1
    assert checked >= 10
