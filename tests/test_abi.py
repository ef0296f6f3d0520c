"""The C-ABI library without a GPU: it loads, exports every symbol the header
declares, and rejects bad arguments with the documented status codes before
touching the device. The KernelFn wrappers refuse CPU tensors (no fallback)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from ako_b200 import _native, kernels

HEADER = Path(__file__).resolve().parent.parent / "include" / "ako_b200.h"


@pytest.fixture(scope="module")
def lib():
    if not _native.LIB_PATH.exists():
        from ako_b200.build import build

        build()
    return _native.lib()


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(ako_b200_\w+)\s*\(", text, re.M)))


def test_header_declares_the_bound_symbols() -> None:
    assert declared_symbols() == sorted(_native.SIGNATURES)


def test_library_exports_every_declared_symbol(lib) -> None:
    raw = ctypes.CDLL(str(_native.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(raw, name), name


def test_abi_version(lib) -> None:
    assert lib.ako_b200_abi_version() == _native.ABI_VERSION == 2


def test_status_strings(lib) -> None:
    assert lib.ako_b200_status_string(0) == b"AKO_B200_OK"
    assert lib.ako_b200_status_string(3) == b"AKO_B200_ERR_CUDA"
    assert lib.ako_b200_status_string(99) == b"AKO_B200_ERR_UNKNOWN"


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


def test_launch_override_validation(lib) -> None:
    assert lib.ako_b200_rmsnorm_set_launch(1, 128, 4) == 0
    assert lib.ako_b200_rmsnorm_set_launch(4, 128, 4) == 0
    assert lib.ako_b200_rmsnorm_set_launch(0, 0, 0) == 0
    assert lib.ako_b200_rmsnorm_set_launch(1, 96, 3) == 1
    assert lib.ako_b200_rmsnorm_set_launch(3, 128, 4) == 1
    assert lib.ako_b200_rmsnorm_set_launch(2, 1024, 8) == 1


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


def test_pdl_switch_returns_previous_setting(lib) -> None:
    assert lib.ako_b200_set_pdl(0) == 1  # on by default
    assert lib.ako_b200_set_pdl(5) == 0
    assert lib.ako_b200_set_pdl(1) == 1


def test_rope_launch_override_validation(lib) -> None:
    assert lib.ako_b200_rope_set_launch(2) == 0
    assert lib.ako_b200_rope_set_launch(0) == 0
    assert lib.ako_b200_rope_set_launch(3) == 1


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


def test_staging_hook_validation(lib) -> None:
    assert lib.ako_b200_rmsnorm_set_staging(2, 4, 2) == 0
    assert lib.ako_b200_rmsnorm_set_staging(0, 0, 0) == 0
    assert lib.ako_b200_rmsnorm_set_staging(3, 0, 0) == 0
    assert lib.ako_b200_rmsnorm_set_staging(0, 0, 0) == 0
    assert lib.ako_b200_rmsnorm_set_staging(4, 0, 0) == 1
    assert lib.ako_b200_rmsnorm_set_staging(2, 9, 1) == 1
    assert lib.ako_b200_take_device_status(None) == 1


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
