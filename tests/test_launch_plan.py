"""Host-side launch choices of the RMSNorm, RoPE and SwiGLU entry points (no
GPU needed).

``ako_b200_rmsnorm_plan``, ``ako_b200_rope_plan`` and ``ako_b200_swiglu_plan``
report the kernel and launch shape a call would get from the built-in choice,
through the same code the launch takes. These cases pin the measured rules: for RMSNorm the tables
for the benchmark's widths, fitted thread counts for widths that are not a
power of two of 16-byte vectors, a warp per row for narrow rows in bulk,
clusters for decode and for 65536-wide fused rows, the staged and chunked
persistent kernels for wide plain 16-bit rows, and the any-width kernel for
unaligned calls; for RoPE the access width (with the 4-byte rule for 8-head
decode calls), heads per thread and CTA extent; for SwiGLU the access width,
CTA size and vectors per thread by problem size and layout.
"""

from __future__ import annotations

import ctypes

import pytest

from ako_b200 import _native

F32, F16, BF16 = 0, 1, 2
ROWS, STAGED, CHUNKED, GENERIC = 0, 1, 2, 3


def plan(rows: int, h: int, dtype: int, residual: bool, aligned: bool = True, lib=None) -> tuple[int, int, int, int]:
    lib = lib or _native.lib()
    out = [ctypes.c_int() for _ in range(4)]
    rc = lib.ako_b200_rmsnorm_plan(rows, h, dtype, int(residual), int(aligned), *(ctypes.byref(o) for o in out))
    assert rc == 0, lib.ako_b200_last_error()
    return tuple(o.value for o in out)


@pytest.fixture(autouse=True)
def _built_in_choice():
    """Overrides live in the measurement build only; reset them around each test."""
    m = _native.measure_lib()
    for f in (lambda: m.ako_b200_rmsnorm_set_launch(0, 0, 0), lambda: m.ako_b200_rmsnorm_set_staging(0, 0, 0),
              lambda: m.ako_b200_swiglu_set_launch(0, 0), lambda: m.ako_b200_rope_set_launch(0),
              lambda: m.ako_b200_swiglu_set_grid(0), lambda: m.ako_b200_swiglu_set_smem(0),
              lambda: m.ako_b200_rmsnorm_set_generic(0)):
        f()
    yield
    m.ako_b200_rmsnorm_set_launch(0, 0, 0)
    m.ako_b200_rmsnorm_set_staging(0, 0, 0)
    m.ako_b200_swiglu_set_launch(0, 0)
    m.ako_b200_swiglu_set_grid(0)
    m.ako_b200_swiglu_set_smem(0)
    m.ako_b200_rmsnorm_set_generic(0)
    m.ako_b200_rope_set_launch(0)


@pytest.mark.parametrize(
    "rows, h, dtype, residual, expected",
    [
        # the benchmark: the headline cell, config 1, config 2 widths
        (32768, 16384, BF16, True, (ROWS, 1, 512, 4)),
        (2048, 4096, F32, False, (ROWS, 1, 256, 4)),
        (8192, 2048, BF16, True, (ROWS, 1, 128, 2)),
        (8192, 4096, F16, True, (ROWS, 1, 256, 2)),
        (8192, 8192, BF16, True, (ROWS, 1, 512, 2)),
        # a few hundred fused rows: two vectors per thread
        (512, 2048, BF16, True, (ROWS, 1, 128, 2)),
        (256, 2048, BF16, True, (ROWS, 1, 256, 1)),
        (256, 4096, F16, True, (ROWS, 1, 256, 2)),
        (512, 4096, BF16, True, (ROWS, 1, 256, 2)),
        (128, 4096, BF16, True, (ROWS, 1, 512, 1)),
        (512, 4096, BF16, False, (ROWS, 1, 256, 2)),
        # decode: latency shapes and clusters
        (1, 4096, BF16, True, (ROWS, 1, 512, 1)),
        (1, 16384, BF16, True, (ROWS, 4, 512, 1)),
        (64, 16384, BF16, True, (ROWS, 4, 256, 2)),
        # fitted thread counts (5120 bf16 = 640 vectors, 4608 = 576)
        (8192, 5120, BF16, True, (ROWS, 1, 320, 2)),
        (8192, 5120, BF16, False, (ROWS, 1, 160, 4)),
        (8192, 4608, BF16, True, (ROWS, 1, 320, 2)),
        (8192, 9216, BF16, False, (ROWS, 1, 320, 4)),
        (8192, 2304, F32, True, (ROWS, 1, 320, 2)),
        # narrow rows in bulk: a warp per row
        (32768, 1024, BF16, False, (ROWS, 1, 32, 4)),
        (4096, 1024, BF16, True, (ROWS, 1, 64, 2)),
        (16384, 1024, BF16, True, (ROWS, 1, 32, 4)),
        (16384, 1536, BF16, False, (ROWS, 1, 32, 8)),
        (8192, 1536, BF16, False, (ROWS, 1, 64, 4)),
        # wide rows: staged (16385-32768 16-bit elements) and chunked (32769-65536)
        (8192, 32768, BF16, False, (STAGED, 1, 1024, 4)),
        (512, 32768, BF16, False, (ROWS, 1, 1024, 4)),
        (8192, 32768, BF16, True, (ROWS, 1, 1024, 4)),
        (512, 65536, F16, False, (CHUNKED, 1, 1024, 8)),
        (512, 65536, BF16, False, (ROWS, 1, 1024, 8)),
        (2048, 65536, BF16, False, (CHUNKED, 1, 1024, 8)),
        (2048, 40960, BF16, False, (CHUNKED, 1, 1024, 8)),
        (8192, 32768, F32, False, (ROWS, 1, 1024, 8)),
        (4096, 65536, BF16, True, (ROWS, 8, 256, 4)),
    ],
)
def test_built_in_choice(rows, h, dtype, residual, expected) -> None:
    assert plan(rows, h, dtype, residual) == expected
    # the measurement build makes the same choice while no override is set
    assert plan(rows, h, dtype, residual, lib=_native.measure_lib()) == expected


def test_unaligned_and_ragged_calls_take_the_any_width_kernel() -> None:
    assert plan(8192, 4096, BF16, True, aligned=False) == (GENERIC, 1, 256, 0)
    assert plan(8192, 4100, BF16, True) == (GENERIC, 1, 256, 0)
    assert plan(8192, 4100, F32, False)[0] == ROWS  # 16400-byte fp32 rows are whole vectors
    # narrow rows take a warp each (plain up to 8704 bytes, fused up to 6144), whatever the row count
    for rows in (1, 7, 65536):
        assert plan(rows, 1001, BF16, False) == (GENERIC, 1, 32, 0)
        assert plan(rows, 3072, BF16, True, aligned=False) == (GENERIC, 1, 32, 0)
        assert plan(rows, 3073, BF16, True, aligned=False) == (GENERIC, 1, 256, 0)
        assert plan(rows, 4100, BF16, False) == (GENERIC, 1, 32, 0)
        assert plan(rows, 2177, F32, False) == (GENERIC, 1, 256, 0)
        assert plan(rows, 1023, F32, True) == (GENERIC, 1, 32, 0)
    assert plan(8, 1537, F32, True) == (GENERIC, 1, 256, 0)
    m = _native.measure_lib()
    assert m.ako_b200_rmsnorm_set_generic(256) == 0
    assert plan(8, 1001, BF16, False, lib=m) == (GENERIC, 1, 256, 0)
    assert m.ako_b200_rmsnorm_set_generic(64) == 1 and m.ako_b200_rmsnorm_set_generic(0) == 0
    assert plan(8, 1001, BF16, False, lib=m) == (GENERIC, 1, 32, 0)


def test_measurement_overrides_are_followed() -> None:
    """The measurement build follows its overrides; the product library,
    which has none, keeps its built-in choice meanwhile."""
    m = _native.measure_lib()
    assert m.ako_b200_rmsnorm_set_launch(2, 512, 4) == 0
    assert plan(8192, 8192, BF16, True, lib=m) == (ROWS, 2, 512, 4)
    assert plan(8192, 8192, BF16, True) == (ROWS, 1, 512, 2)
    # a split into slices of partial 32-vector groups is not taken (8200 / 8 / 2 = 512.5 vectors)
    assert plan(8192, 8200 * 2, BF16, True, lib=m)[1] == 1
    assert m.ako_b200_rmsnorm_set_launch(0, 0, 0) == 0
    assert m.ako_b200_rmsnorm_set_staging(2, 4, 2) == 0
    assert plan(8192, 4096, BF16, True, lib=m) == (STAGED, 1, 256, 2)
    assert plan(8192, 4096, BF16, True) == (ROWS, 1, 256, 2)
    assert m.ako_b200_rmsnorm_set_staging(1, 0, 0) == 0
    assert plan(8192, 32768, BF16, False, lib=m) == (ROWS, 1, 1024, 4)
    assert m.ako_b200_rmsnorm_set_staging(3, 0, 0) == 0
    assert plan(8192, 24576, BF16, False, lib=m) == (CHUNKED, 1, 1024, 4)


def test_invalid_arguments_are_rejected() -> None:
    out = [ctypes.c_int() for _ in range(4)]
    lib = _native.lib()
    assert lib.ako_b200_rmsnorm_plan(8, 4096, 7, 0, 1, *(ctypes.byref(o) for o in out)) == 2
    assert lib.ako_b200_rmsnorm_plan(8, 0, BF16, 0, 1, *(ctypes.byref(o) for o in out)) == 1
    assert lib.ako_b200_rmsnorm_plan(8, 4096, BF16, 0, 1, None, None, None, None) == 1


def swiglu_plan(rows: int, f: int, dtype: int, aligned: bool = True, dense: bool = True, lib=None
                ) -> tuple[int, int, int, int]:
    lib = lib or _native.lib()
    out = [ctypes.c_int() for _ in range(4)]
    rc = lib.ako_b200_swiglu_plan(rows, f, dtype, int(aligned), int(dense), *(ctypes.byref(o) for o in out))
    assert rc == 0, lib.ako_b200_last_error()
    return tuple(o.value for o in out)


@pytest.mark.parametrize(
    "rows, f, dtype, aligned, dense, expected",
    [
        (16384, 14336, BF16, True, True, (16, 256, 2, 2048)),   # 2^24.8 dense vectors: two per thread
        (16384, 14336, BF16, True, False, (16, 256, 2, 1024)),  # packed halves (strided): two, 1024 threads/SM
        (16384, 11008, F16, True, False, (16, 256, 2, 1024)),
        (16384, 14336, F16, True, True, (16, 256, 2, 2048)),    # fp16 dense: a full budget, four resident
        (16384, 5632, BF16, True, False, (16, 256, 1, 2048)),   # below 2^24 vectors
        (2048, 11008, F16, True, True, (16, 256, 1, 2048)),
        (64, 14336, BF16, True, True, (16, 128, 1, 2048)),      # decode rows: 128-thread CTAs
        (1, 14336, F16, True, True, (4, 128, 1, 2048)),         # decode-sized: two elements per thread
        (2, 16384, F32, True, True, (4, 128, 1, 2048)),         # 2^15 elements, the limit
        (1, 32776, BF16, True, True, (16, 128, 1, 2048)),       # just above it
        (7, 100, BF16, True, True, (2, 256, 4, 2048)),          # 200-byte rows: element accesses
        (8, 4096, BF16, False, True, (2, 256, 4, 2048)),        # unaligned operands
    ],
)
def test_swiglu_built_in_choice(rows, f, dtype, aligned, dense, expected) -> None:
    assert swiglu_plan(rows, f, dtype, aligned, dense) == expected


def test_swiglu_override_is_followed() -> None:
    m = _native.measure_lib()
    assert m.ako_b200_swiglu_set_launch(64, 2) == 0
    assert swiglu_plan(2048, 11008, BF16, lib=m) == (16, 64, 2, 2048)
    assert swiglu_plan(1, 5632, BF16, lib=m) == (16, 64, 2, 2048)  # an override also skips the decode-sized path
    assert m.ako_b200_swiglu_set_grid(1536) == 0
    assert swiglu_plan(2048, 11008, BF16, lib=m) == (16, 64, 2, 1536)
    assert m.ako_b200_swiglu_set_grid(4096) == 0
    assert swiglu_plan(2048, 11008, BF16, lib=m) == (16, 64, 2, 4096)
    assert m.ako_b200_swiglu_set_grid(100) == 1 and m.ako_b200_swiglu_set_grid(8256) == 1
    assert m.ako_b200_swiglu_set_grid(0) == 0
    assert m.ako_b200_swiglu_set_smem(48 * 1024) == 0 and m.ako_b200_swiglu_set_smem(48 * 1024 + 1) == 1
    assert m.ako_b200_swiglu_set_smem(-1) == 1 and m.ako_b200_swiglu_set_smem(0) == 0
    assert swiglu_plan(2048, 11008, BF16) == (16, 256, 1, 2048)


def rope_plan(b: int, s: int, h: int, d: int, style: int, dtype: int, lib=None) -> tuple[int, int, int, int, int]:
    lib = lib or _native.lib()
    out = [ctypes.c_int() for _ in range(5)]
    rc = lib.ako_b200_rope_plan(b, s, h, d, style, dtype, *(ctypes.byref(o) for o in out))
    assert rc == 0, lib.ako_b200_last_error()
    return tuple(o.value for o in out)


NEOX, INTERLEAVED = 0, 1


@pytest.mark.parametrize(
    "shape, style, dtype, expected",
    [
        ((32, 4096, 32, 128), NEOX, BF16, (16, 1, 8, 32, 1)),        # config 3 q: 8 threads per head row
        ((32, 4096, 8, 128), NEOX, BF16, (16, 1, 8, 8, 4)),          # config 3 k: 4 positions per CTA
        ((8, 512, 32, 128), INTERLEAVED, BF16, (16, 2, 8, 16, 2)),   # interleaved: two heads per thread
        ((16, 4096, 32, 128), NEOX, F32, (16, 1, 16, 16, 1)),
        ((1, 1, 32, 128), NEOX, BF16, (16, 1, 8, 32, 1)),            # 32-head decode keeps 16 bytes
        ((8, 1, 8, 128), NEOX, BF16, (4, 1, 32, 8, 1)),              # 8-head decode: 4-byte accesses
        ((32, 1, 8, 128), NEOX, F16, (4, 1, 32, 8, 1)),
        ((1, 1, 8, 128), NEOX, F32, (16, 1, 16, 8, 1)),              # fp32: 4 bytes is one element
        ((8, 512, 32, 100), NEOX, BF16, (4, 1, 25, 10, 1)),          # half of 50: 4-byte accesses
        ((8, 512, 32, 98), NEOX, BF16, (2, 1, 49, 5, 1)),            # odd half: a pair per thread
    ],
)
def test_rope_built_in_choice(shape, style, dtype, expected) -> None:
    assert rope_plan(*shape, style, dtype) == expected


def test_rope_override_and_errors() -> None:
    m = _native.measure_lib()
    assert m.ako_b200_rope_set_launch(2) == 0
    assert rope_plan(32, 4096, 32, 128, NEOX, BF16, lib=m) == (16, 2, 8, 16, 2)
    assert rope_plan(32, 4096, 32, 128, NEOX, BF16) == (16, 1, 8, 32, 1)
    lib = _native.lib()
    out = [ctypes.c_int() for _ in range(5)]
    assert lib.ako_b200_rope_plan(1, 1, 8, 127, NEOX, BF16, *(ctypes.byref(o) for o in out)) == 1
    assert lib.ako_b200_rope_plan(1, 1, 8, 128, 5, BF16, *(ctypes.byref(o) for o in out)) == 1
    assert lib.ako_b200_rope_plan(1, 1, 8, 128, NEOX, 9, *(ctypes.byref(o) for o in out)) == 2


@pytest.mark.parametrize("dtype", (F32, F16, BF16))
@pytest.mark.parametrize("residual", (False, True))
def test_every_rmsnorm_plan_covers_its_row(dtype: int, residual: bool) -> None:
    """Over every 16-byte-aligned width up to 65536 and a spread of row counts,
    the chosen launch holds the whole row: a cluster of CTAs of threads x
    vectors (or the persistent kernels' 1024 or 256 threads) spans at least
    the row's 16-byte vectors, and a row-resident CTA has at most 1024
    threads. (A shape that fell short would leave the row's tail unwritten.)"""
    vec = 4 if dtype == F32 else 8
    for rows in (1, 8, 33, 64, 65, 512, 513, 1024, 8192, 16384, 40000):
        for h in range(vec, 65536 + 1, vec):
            kernel, cluster, threads, vectors = plan(rows, h, dtype, residual)
            nvec = h // vec
            if kernel == GENERIC:
                continue
            assert cluster * threads * vectors >= nvec, (rows, h, kernel, cluster, threads, vectors)
            assert threads <= 1024 and cluster in (1, 2, 4, 8)
            # the fixed summation order: whole warps per row slice, slices of whole 32-vector groups
            assert threads % 32 == 0 and nvec % (32 * cluster) == 0 if cluster > 1 else threads % 32 == 0, (
                rows, h, cluster, threads)
            if kernel in (STAGED, CHUNKED):
                assert not residual or kernel == STAGED
                assert cluster == 1


@pytest.mark.parametrize("dtype", (F32, F16, BF16))
def test_every_rope_plan_fits_its_kernel(dtype: int) -> None:
    """Over every even head size up to 512, a spread of head counts and
    position counts, and both styles: the CTA stays within the kernels'
    256-thread launch bound, and in the vector kernel a head row's threads
    times the pairs each rotates per half equal the half head size."""
    es = 4 if dtype == F32 else 2
    for d in range(2, 513, 2):
        for heads in (1, 3, 8, 32, 40, 64):
            for b, s in ((1, 1), (8, 1), (2, 37), (4, 4096)):
                for style in (NEOX, INTERLEAVED):
                    access, hpt, bx, by, bz = rope_plan(b, s, heads, d, style, dtype)
                    assert 1 <= bx * by * bz <= 256, (d, heads, b, s, style)
                    assert bz <= b * s and by * hpt >= 1
                    if access // es >= 2:  # the vector kernel (the pair-per-thread kernel loops over the row)
                        assert bx * (access // es) == d // 2, (d, heads, b, s, style, access, bx)
                    else:
                        assert access == es and bx == min(d // 2, 256), (d, heads, b, s, style, access, bx)
