"""The C-ABI libraries without a GPU: each loads and exports every symbol its
header declares (the product library none of the measurement overrides), and
rejects bad arguments with the documented status codes before touching the
device. The KernelFn wrappers refuse CPU tensors (no fallback)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from ako_b200 import _native, kernels

INCLUDE = Path(__file__).resolve().parent.parent / "include"
HEADER = INCLUDE / "ako_b200.h"
MEASURE_HEADER = INCLUDE / "ako_b200_measure.h"


def _built() -> None:
    if not (_native.LIB_PATH.exists() and _native.MEASURE_LIB_PATH.exists()):
        from ako_b200.build import build

        build()


@pytest.fixture(scope="module")
def lib():
    _built()
    return _native.lib()


@pytest.fixture(scope="module")
def mlib():
    _built()
    return _native.measure_lib()


def declared_symbols(header: Path = HEADER) -> list[str]:
    text = header.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+|unsigned\s+)?\w+\*?\s+\*?(ako_b200_\w+)\s*\(", text, re.M)))


def _exported(path: Path) -> set[str]:
    raw = ctypes.CDLL(str(path))
    return {n for n in [*_native.SIGNATURES, *_native.MEASURE_SIGNATURES] if hasattr(raw, n)}


def test_headers_declare_the_bound_symbols() -> None:
    assert declared_symbols(HEADER) == sorted(_native.SIGNATURES)
    assert declared_symbols(MEASURE_HEADER) == sorted(_native.MEASURE_SIGNATURES)


def test_library_exports_every_declared_symbol(lib) -> None:
    raw = ctypes.CDLL(str(_native.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(raw, name), name


def test_product_library_has_no_measurement_overrides(lib) -> None:
    """Forced shapes, kernels, launch modes and wait limits exist only in the
    measurement build: the product library exports none of them."""
    assert _exported(_native.LIB_PATH) == set(_native.SIGNATURES)


def test_measurement_library_exports_both_headers(mlib) -> None:
    assert _exported(_native.MEASURE_LIB_PATH) == set(_native.SIGNATURES) | set(_native.MEASURE_SIGNATURES)
    assert set(declared_symbols(HEADER)) | set(declared_symbols(MEASURE_HEADER)) <= _exported(_native.MEASURE_LIB_PATH)


def test_abi_version(lib, mlib) -> None:
    assert lib.ako_b200_abi_version() == mlib.ako_b200_abi_version() == _native.ABI_VERSION == 4


def test_status_strings(lib) -> None:
    assert lib.ako_b200_status_string(0) == b"AKO_B200_OK"
    assert lib.ako_b200_status_string(3) == b"AKO_B200_ERR_CUDA"
    assert lib.ako_b200_status_string(4) == b"AKO_B200_ERR_WAIT_EXPIRED"
    assert lib.ako_b200_status_string(99) == b"AKO_B200_ERR_UNKNOWN"


def test_device_status_without_any_persistent_launch(lib) -> None:
    """No persistent kernel has run in this process: the status is 0 and the
    call needs no device."""
    value = ctypes.c_int(7)
    assert lib.ako_b200_take_device_status(ctypes.byref(value)) == 0 and value.value == 0
    assert lib.ako_b200_take_device_status(None) == 1


def test_rmsnorm_argument_errors(lib) -> None:
    p = 16  # never dereferenced: every call below fails before a launch
    assert lib.ako_b200_rmsnorm(p, 8, p, 0, p, 8, 4, 8, 1e-6, 7, None) == _native.ERR_UNSUPPORTED_DTYPE
    assert b"dtype" in lib.ako_b200_last_error()
    assert lib.ako_b200_rmsnorm(p, 8, p, 9, p, 8, 4, 8, 1e-6, 0, None) == _native.ERR_UNSUPPORTED_DTYPE
    assert lib.ako_b200_rmsnorm(p, 8, p, 0, p, 8, -1, 8, 1e-6, 0, None) == _native.ERR_INVALID_ARGUMENT
    assert lib.ako_b200_rmsnorm(p, 8, p, 0, p, 8, 4, 0, 1e-6, 0, None) == _native.ERR_INVALID_ARGUMENT
    assert b"hidden_dim" in lib.ako_b200_last_error()
    assert lib.ako_b200_rmsnorm(None, 8, p, 0, p, 8, 4, 8, 1e-6, 0, None) == _native.ERR_INVALID_ARGUMENT
    assert b"x is a null pointer" in lib.ako_b200_last_error()
    assert lib.ako_b200_rmsnorm(p, 4, p, 0, p, 8, 4, 8, 1e-6, 0, None) == _native.ERR_INVALID_ARGUMENT
    assert b"row stride" in lib.ako_b200_last_error()
    # No rows: nothing to do, success without a launch.
    assert lib.ako_b200_rmsnorm(None, 0, None, 0, None, 0, 0, 8, 1e-6, 2, None) == _native.OK
    assert lib.ako_b200_last_error() == b""


def test_residual_rope_swiglu_argument_errors(lib) -> None:
    p = 16
    assert lib.ako_b200_rmsnorm_residual(p, 8, None, 8, p, 0, p, 8, p, 8, 2, 8, 1e-5, 2, None) == 1
    assert b"residual is a null pointer" in lib.ako_b200_last_error()
    rope = lib.ako_b200_rope
    assert rope(p, 0, 0, 0, p, p, 4, p, 0, 0, 0, 1, 1, 1, 8, 5, 2, None) == 1  # style
    assert rope(p, 0, 0, 0, p, p, 4, p, 0, 0, 0, 1, 1, 1, 7, 0, 2, None) == 1  # odd head_dim
    assert rope(p, 0, 0, 0, p, p, 4, p, 0, 0, 0, 1, 1, 1, 8, 0, 3, None) == 2  # dtype
    assert rope(p, 0, 0, 0, p, p, 2, p, 0, 0, 0, 1, 2, 1, 8, 0, 2, None) == 1  # table stride < D/2
    assert rope(None, 0, 0, 0, None, None, 0, None, 0, 0, 0, 0, 4, 2, 8, 0, 2, None) == 0  # empty batch
    qk = lib.ako_b200_rope_qk
    assert qk(p, 0, 0, 0, p, 0, 0, 0, p, p, 4, p, 0, 0, 0, p, 0, 0, 0, 1, 1, 2, 1, 8, 7, 2, None) == 1  # style
    assert qk(p, 0, 0, 0, p, 0, 0, 0, p, p, 4, p, 0, 0, 0, p, 0, 0, 0, 1, 1, -1, 1, 8, 0, 2, None) == 1  # heads
    assert qk(p, 0, 0, 0, None, 0, 0, 0, p, p, 4, p, 0, 0, 0, None, 0, 0, 0, 1, 1, 2, 1, 8, 0, 2, None) == 1
    assert qk(None, 0, 0, 0, None, 0, 0, 0, p, p, 4, None, 0, 0, 0, None, 0, 0, 0, 1, 1, 0, 0, 8, 0, 2, None) == 0
    assert lib.ako_b200_swiglu(p, 8, p, 8, p, 8, 2, 8, 5, None) == 2
    assert lib.ako_b200_swiglu(p, 4, p, 8, p, 8, 2, 8, 2, None) == 1
    assert lib.ako_b200_swiglu(None, 0, None, 0, None, 0, 0, 8, 2, None) == 0


def test_launch_override_validation(mlib) -> None:
    assert mlib.ako_b200_rmsnorm_set_launch(1, 128, 4) == 0
    assert mlib.ako_b200_rmsnorm_set_launch(4, 128, 4) == 0
    assert mlib.ako_b200_rmsnorm_set_launch(0, 0, 0) == 0
    assert mlib.ako_b200_rmsnorm_set_launch(1, 96, 3) == 1
    assert mlib.ako_b200_rmsnorm_set_launch(3, 128, 4) == 1
    assert mlib.ako_b200_rmsnorm_set_launch(2, 1024, 8) == 1


@pytest.mark.parametrize(
    "call",
    [
        lambda: kernels.rmsnorm_cuda_sm100(torch.randn(2, 8), torch.ones(8)),
        lambda: kernels.rmsnorm_residual_cuda_sm100(torch.randn(2, 8), torch.randn(2, 8), torch.ones(8)),
        lambda: kernels.rope_cuda_sm100(torch.randn(1, 2, 1, 8), torch.ones(2, 4), torch.zeros(2, 4)),
        lambda: kernels.swiglu_cuda_sm100(torch.randn(2, 8), torch.randn(2, 8)),
        lambda: kernels.rope_qk_cuda_sm100(torch.randn(1, 2, 4, 8), torch.randn(1, 2, 2, 8), torch.ones(2, 4),
                                           torch.zeros(2, 4)),
    ],
    ids=["rmsnorm", "rmsnorm_residual", "rope", "swiglu", "rope_qk"],
)
def test_wrappers_refuse_cpu_tensors(call) -> None:
    with pytest.raises(ValueError, match="requires a CUDA tensor"):
        call()


def test_wrapper_shape_and_style_errors() -> None:
    with pytest.raises(ValueError, match="Unknown RoPE style"):
        kernels.rope_cuda_sm100(torch.randn(1, 2, 1, 8), torch.ones(2, 4), torch.zeros(2, 4), "bogus")
    with pytest.raises(ValueError):
        kernels.rmsnorm_residual_cuda_sm100(torch.randn(2, 8), torch.randn(2, 4), torch.ones(8))
    with pytest.raises(ValueError):
        kernels.swiglu_cuda_sm100(torch.randn(2, 8), torch.randn(2, 16))


def test_missing_library_fails_loudly(monkeypatch, tmp_path) -> None:
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setenv("AKO_B200_LIB", str(tmp_path / "absent.so"))
    with pytest.raises(_native.NativeLibraryError, match="not built"):
        _native.lib()


def test_measurement_block_routes_only_its_own_thread(lib, mlib) -> None:
    """Inside ``measurement()`` this thread's wrappers call the measurement
    build; other threads, and this one afterwards, call the product library."""
    import threading

    seen = {}
    assert _native.active() is lib
    with _native.measurement() as m:
        assert m is mlib and _native.active() is mlib
        t = threading.Thread(target=lambda: seen.setdefault("other", _native.active()))
        t.start()
        t.join()
    assert seen["other"] is lib and _native.active() is lib


def test_pdl_switch_returns_previous_setting(mlib) -> None:
    assert mlib.ako_b200_set_pdl(0) == 1  # on by default
    assert mlib.ako_b200_set_pdl(5) == 0
    assert mlib.ako_b200_set_pdl(1) == 1


def test_wait_limit_switch_returns_previous_setting(mlib) -> None:
    assert mlib.ako_b200_measure_set_wait_polls(0) == 1 << 24
    assert mlib.ako_b200_measure_set_wait_polls(1 << 24) == 0


def test_rope_launch_override_validation(mlib) -> None:
    assert mlib.ako_b200_rope_set_launch(2) == 0
    assert mlib.ako_b200_rope_set_launch(0) == 0
    assert mlib.ako_b200_rope_set_launch(3) == 1


def _fastdiv(d: int) -> tuple[int, int]:
    """Host half of the kernels' FastDiv (csrc/common.cuh), restated."""
    l = 0
    while (1 << l) < d:
        l += 1
    m = ((1 << 32) * ((1 << l) - d)) // d + 1
    assert 0 < m < (1 << 32)
    return m, l


@pytest.mark.parametrize("d", [1, 2, 3, 5, 7, 100, 704, 1376, 1792, 4095, 4096, 4097, 65535, 2**31 - 1, 2**31,
                               2**31 + 1, 2**32 - 1])
def test_multiply_high_division_is_exact(d: int) -> None:
    """q = (mulhi(n, m) + n) >> l equals n // d over boundary and random n < 2^32."""
    import random

    m, l = _fastdiv(d)
    rnd = random.Random(d)
    ns = [0, 1, d - 1, d, d + 1, 2**32 - 1, 2**32 - d, (2**32 - 1) // d * d, (2**32 - 1) // d * d - 1]
    ns += [rnd.randrange(2**32) for _ in range(2000)] + [k * d + r for k in (1, 7, 1000) for r in (0, d - 1)]
    for n in ns:
        if 0 <= n < 2**32:
            assert ((((n * m) >> 32) + n) >> l) == n // d, (n, d)


def test_staging_hook_validation(mlib) -> None:
    assert mlib.ako_b200_rmsnorm_set_staging(2, 4, 2) == 0
    assert mlib.ako_b200_rmsnorm_set_staging(0, 0, 0) == 0
    assert mlib.ako_b200_rmsnorm_set_staging(3, 0, 0) == 0
    assert mlib.ako_b200_rmsnorm_set_staging(0, 0, 0) == 0
    assert mlib.ako_b200_rmsnorm_set_staging(4, 0, 0) == 1
    assert mlib.ako_b200_rmsnorm_set_staging(2, 9, 1) == 1
    assert mlib.ako_b200_take_device_status(None) == 1


def test_host_pipeline_chunking_and_argument_checks() -> None:
    """The host-buffer pipeline's chunk arithmetic (one launch per chunk of
    32 MB per operand) and its argument errors, all decided before any GPU
    work."""
    from ako_b200 import host

    assert host.DEFAULT_CHUNK_BYTES == 32 << 20
    assert host.launches_per_call(32768, 16384, 2) == 32  # 1024 rows of 32 KB per chunk
    assert host.launches_per_call(1000, 16384, 2) == 1
    assert host.launches_per_call(1025, 16384, 2, chunk_rows=1024) == 2
    assert host.launches_per_call(0, 4096, 2) == 0
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="Shape mismatch"):
        host.rmsnorm_residual_host(x, torch.zeros(4, 9, dtype=torch.bfloat16), torch.ones(8))
    with pytest.raises(ValueError, match="supports float32/float16/bfloat16"):
        host.rmsnorm_residual_host(x.to(torch.int32), x.to(torch.int32), torch.ones(8))
    with pytest.raises(ValueError, match="weight must live on the target CUDA device"):
        host.rmsnorm_residual_host(x, x, torch.ones(8))


def test_host_slot_capacity_is_bounded() -> None:
    """Calls of many row counts share few slot sizes: the chunk, or the next
    power of two at or above a smaller call's rows."""
    from ako_b200 import host

    caps = {host.slot_capacity(rows, 1024) for rows in range(1, 5000)}
    assert caps == {1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024}
    assert host.slot_capacity(1000, 1024) == 1024 and host.slot_capacity(5, 4) == 4
    assert host.MAX_SLOT_SETS == 4


def test_host_pipeline_checks_weight_and_outputs() -> None:
    from ako_b200 import host

    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    meta_w = torch.ones(16, device="meta")[::2]  # a strided (8,) view: accepted as a copy, never as-is
    assert host._host_weight(meta_w, 8, "f").stride(0) == 1
    with pytest.raises(ValueError, match="Expected weight of shape"):
        host._host_weight(torch.ones(9), 8, "f")
    with pytest.raises(ValueError, match="hidden_dim <= 65536"):
        host._host_weight(torch.ones(65537), 65537, "f")
    dev_w = torch.ones(8, device="meta")
    for bad in (torch.zeros(4, 9, dtype=torch.bfloat16), torch.zeros(4, 8, dtype=torch.float32)):
        with pytest.raises(ValueError, match="y_out must be a host tensor"):
            host.rmsnorm_residual_host(x, x, dev_w, device="meta", y_out=bad)
