"""ctypes binding of ``libako_b200.so`` (the C ABI declared in ``include/ako_b200.h``).

The library is built in-tree by :mod:`ako_b200.build`. There is no fallback:
if the library is missing or does not export a declared symbol, :func:`lib`
raises, and every kernel wrapper with it.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libako_b200.so"

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
    "ako_b200_rmsnorm_set_launch": (_c_int, [_c_int, _c_int, _c_int]),
    "ako_b200_rope_plan": (_c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _c_int, _c_int,
                                    ctypes.POINTER(_c_int), ctypes.POINTER(_c_int), ctypes.POINTER(_c_int),
                                    ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "ako_b200_swiglu_plan": (_c_int, [ctypes.c_int64, ctypes.c_int64, _c_int, _c_int, _c_int,
                                      ctypes.POINTER(_c_int), ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "ako_b200_rmsnorm_plan": (_c_int, [ctypes.c_int64, ctypes.c_int64, _c_int, _c_int, _c_int,
                                       ctypes.POINTER(_c_int), ctypes.POINTER(_c_int), ctypes.POINTER(_c_int),
                                       ctypes.POINTER(_c_int)]),
    "ako_b200_rope_set_launch": (_c_int, [_c_int]),
    "ako_b200_swiglu_set_launch": (_c_int, [_c_int, _c_int]),
    "ako_b200_set_pdl": (_c_int, [_c_int]),
    "ako_b200_rmsnorm_set_staging": (_c_int, [_c_int, _c_int, _c_int]),
    "ako_b200_take_device_status": (_c_int, [ctypes.POINTER(ctypes.c_int)]),
}

ABI_VERSION = 2

# Status codes (ako_b200_status).
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED_DTYPE = 2
ERR_CUDA = 3

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing, stale or incomplete."""


def lib() -> ctypes.CDLL:
    """Load (once) and return the library with argtypes set for every symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("AKO_B200_LIB", LIB_PATH))
        if not path.exists():
            raise NativeLibraryError(
                f"{path} is not built; run `python -m ako_b200.build` (nvcc, sm_100a)"
            )
        handle = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in SIGNATURES.items():
            try:
                fn = getattr(handle, name)
            except AttributeError as exc:
                raise NativeLibraryError(f"{path} does not export {name}") from exc
            fn.restype = restype
            fn.argtypes = argtypes
        version = handle.ako_b200_abi_version()
        if version != ABI_VERSION:
            raise NativeLibraryError(f"{path} has ABI {version}, expected {ABI_VERSION}; rebuild it")
        _lib = handle
    return _lib


def last_error() -> str:
    return lib().ako_b200_last_error().decode(errors="replace")


def raise_for_status(status: int, op: str) -> None:
    """Turn a non-zero status into the exception type AKO's dispatcher expects."""
    if status == OK:
        return
    message = last_error() or lib().ako_b200_status_string(status).decode()
    if status in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED_DTYPE):
        raise ValueError(f"{op}: {message}")
    raise RuntimeError(f"{op}: {message}")


def take_device_status() -> int:
    """Read and clear the kernels' device status word (0 = no bounded wait ran out)."""
    value = ctypes.c_int(0)
    raise_for_status(lib().ako_b200_take_device_status(ctypes.byref(value)), "take_device_status")
    return value.value
