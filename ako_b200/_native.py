"""ctypes binding of ``libako_b200.so`` (the C ABI declared in ``include/ako_b200.h``)
and of its measurement build ``libako_b200_measure.so`` (``include/ako_b200_measure.h``).

Both are built in-tree by :mod:`ako_b200.build`. There is no fallback: if a
library is missing or does not export a declared symbol, :func:`lib` (or
:func:`measure_lib`) raises, and every kernel wrapper with it.

The kernel wrappers call :func:`active`, which is the product library unless
the calling thread is inside :func:`measurement`: sweeps and tests use that
to run the same wrappers through the measurement build after forcing a
launch shape there. Nothing reaches the measurement build otherwise.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
import threading
from collections.abc import Iterator
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libako_b200.so"
MEASURE_LIB_PATH = Path(__file__).resolve().parent / "libako_b200_measure.so"

_c_int = ctypes.c_int
_c_i64 = ctypes.c_int64
_c_dbl = ctypes.c_double
_c_ptr = ctypes.c_void_p

#: Exported symbol -> (restype, argtypes); mirrors include/ako_b200.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ako_b200_abi_version": (_c_int, []),
    "ako_b200_status_string": (ctypes.c_char_p, [_c_int]),
    "ako_b200_last_error": (ctypes.c_char_p, []),
    "ako_b200_rmsnorm": (
        _c_int,
        [_c_ptr, _c_i64, _c_ptr, _c_int, _c_ptr, _c_i64, _c_i64, _c_i64, _c_dbl, _c_int, _c_ptr],
    ),
    "ako_b200_rmsnorm_residual": (
        _c_int,
        [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_int, _c_ptr, _c_i64, _c_ptr, _c_i64,
         _c_i64, _c_i64, _c_dbl, _c_int, _c_ptr],
    ),
    "ako_b200_rope": (
        _c_int,
        [_c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64,
         _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_ptr],
    ),
    "ako_b200_rope_qk": (
        _c_int,
        [_c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_i64,
         _c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64,
         _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_ptr],
    ),
    "ako_b200_swiglu": (
        _c_int,
        [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64, _c_int, _c_ptr],
    ),
    "ako_b200_rope_plan": (_c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _c_int, _c_int,
                                    ctypes.POINTER(_c_int), ctypes.POINTER(_c_int), ctypes.POINTER(_c_int),
                                    ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "ako_b200_swiglu_plan": (_c_int, [ctypes.c_int64, ctypes.c_int64, _c_int, _c_int, _c_int,
                                      ctypes.POINTER(_c_int), ctypes.POINTER(_c_int), ctypes.POINTER(_c_int),
                                      ctypes.POINTER(_c_int)]),
    "ako_b200_rmsnorm_plan": (_c_int, [ctypes.c_int64, ctypes.c_int64, _c_int, _c_int, _c_int,
                                       ctypes.POINTER(_c_int), ctypes.POINTER(_c_int), ctypes.POINTER(_c_int),
                                       ctypes.POINTER(_c_int)]),
    "ako_b200_take_device_status": (_c_int, [ctypes.POINTER(ctypes.c_int)]),
}

#: Symbols only the measurement build exports; mirrors include/ako_b200_measure.h.
MEASURE_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ako_b200_rmsnorm_set_launch": (_c_int, [_c_int, _c_int, _c_int]),
    "ako_b200_rmsnorm_set_staging": (_c_int, [_c_int, _c_int, _c_int]),
    "ako_b200_rmsnorm_set_generic": (_c_int, [_c_int]),
    "ako_b200_measure_set_wait_polls": (ctypes.c_uint, [ctypes.c_uint]),
    "ako_b200_rope_set_launch": (_c_int, [_c_int]),
    "ako_b200_swiglu_set_launch": (_c_int, [_c_int, _c_int]),
    "ako_b200_swiglu_set_grid": (_c_int, [_c_int]),
    "ako_b200_swiglu_set_smem": (_c_int, [_c_int]),
    "ako_b200_set_pdl": (_c_int, [_c_int]),
}

ABI_VERSION = 4

# Status codes (ako_b200_status).
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED_DTYPE = 2
ERR_CUDA = 3
ERR_WAIT_EXPIRED = 4

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_measure_lib: ctypes.CDLL | None = None
_local = threading.local()


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing, stale or incomplete."""


def _load(path: Path, signatures: dict[str, tuple[object, list[object]]]) -> ctypes.CDLL:
    if not path.exists():
        raise NativeLibraryError(f"{path} is not built; run `python -m ako_b200.build` (nvcc, sm_100a)")
    handle = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in signatures.items():
        try:
            fn = getattr(handle, name)
        except AttributeError as exc:
            raise NativeLibraryError(f"{path} does not export {name}") from exc
        fn.restype = restype
        fn.argtypes = argtypes
    version = handle.ako_b200_abi_version()
    if version != ABI_VERSION:
        raise NativeLibraryError(f"{path} has ABI {version}, expected {ABI_VERSION}; rebuild it")
    return handle


def lib() -> ctypes.CDLL:
    """Load (once) and return the product library with argtypes set for every symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            _lib = _load(Path(os.environ.get("AKO_B200_LIB", LIB_PATH)), SIGNATURES)
    return _lib


def measure_lib() -> ctypes.CDLL:
    """Load (once) and return the measurement build (product symbols plus overrides)."""
    global _measure_lib
    if _measure_lib is not None:
        return _measure_lib
    with _lock:
        if _measure_lib is None:
            _measure_lib = _load(MEASURE_LIB_PATH, {**SIGNATURES, **MEASURE_SIGNATURES})
    return _measure_lib


def active() -> ctypes.CDLL:
    """The library the kernel wrappers call on this thread (the product library
    unless inside :func:`measurement`)."""
    override = getattr(_local, "lib", None)
    return override if override is not None else lib()


@contextlib.contextmanager
def measurement() -> Iterator[ctypes.CDLL]:
    """Route this thread's kernel-wrapper calls through the measurement build.

    Yields that library, whose override setters (``include/ako_b200_measure.h``)
    then apply to the calls made inside the block. The overrides themselves
    are process-wide settings of the measurement library; the block restores
    none of them.
    """
    prev = getattr(_local, "lib", None)
    _local.lib = measure_lib()
    try:
        yield _local.lib
    finally:
        _local.lib = prev


def last_error() -> str:
    return active().ako_b200_last_error().decode(errors="replace")


def raise_for_status(status: int, op: str) -> None:
    """Turn a non-zero status into the exception type AKO's dispatcher expects
    (``ValueError`` for arguments, ``RuntimeError`` otherwise)."""
    if status == OK:
        return
    message = last_error() or active().ako_b200_status_string(status).decode()
    if status in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED_DTYPE):
        raise ValueError(f"{op}: {message}")
    raise RuntimeError(f"{op}: {message}")


def take_device_status() -> int:
    """Synchronize, then read and clear the persistent kernels' status word on
    this thread's active library (0: no bounded wait ran out; 1: one did, its
    rows hold NaN, and calls were refused until now)."""
    value = ctypes.c_int(0)
    raise_for_status(active().ako_b200_take_device_status(ctypes.byref(value)), "take_device_status")
    return value.value
