"""ctypes binding of the C oracle (``oracle/ako_oracle.c``) — TEST INFRASTRUCTURE ONLY.

Imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py``; never by the ``ako_b200`` package. Arrays follow the storage
conventions of :mod:`oracle.ako_oracle` (bfloat16 as ``uint16`` bits).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

from oracle.ako_oracle import BF16, F16, F32, storage_dtype

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "_build" / "libako_oracle.so"
_CODE = {F32: 0, F16: 1, BF16: 2}
_lib: ctypes.CDLL | None = None


def build() -> Path:
    """Compile the C oracle with its Makefile (gcc)."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        handle = ctypes.CDLL(str(LIB_PATH))
        p, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        handle.ako_oracle_rmsnorm.argtypes = [p, p, i32, p, i64, i64, f32, i32, i32]
        handle.ako_oracle_rmsnorm_residual.argtypes = [p, p, p, i32, p, p, i64, i64, f32, i32, i32]
        handle.ako_oracle_rmsnorm_fixed_order.argtypes = [p, p, p, i32, p, p, i64, i64, f32, i32, i32]
        handle.ako_oracle_rope.argtypes = [p, p, p, p, i64, i64, i64, i64, i32, i32, i32]
        handle.ako_oracle_swiglu.argtypes = [p, p, p, i64, i64, i32, i32]
        _lib = handle
    return _lib


def default_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def _c(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a)


def rmsnorm(x, w, eps, dtype, w_dtype=None, threads=None):
    x, w = _c(x), _c(w)
    y = np.empty_like(x)
    h = x.shape[-1]
    lib().ako_oracle_rmsnorm(x.ctypes.data, w.ctypes.data, _CODE[w_dtype or dtype], y.ctypes.data,
                             x.size // h, h, float(eps), _CODE[dtype], threads or default_threads())
    return y


def rmsnorm_residual(x, r, w, eps, dtype, w_dtype=None, threads=None):
    x, r, w = _c(x), _c(r), _c(w)
    y = np.empty_like(x)
    ro = np.empty_like(x)
    h = x.shape[-1]
    lib().ako_oracle_rmsnorm_residual(x.ctypes.data, r.ctypes.data, w.ctypes.data, _CODE[w_dtype or dtype],
                                      y.ctypes.data, ro.ctypes.data, x.size // h, h, float(eps), _CODE[dtype],
                                      threads or default_threads())
    return y, ro


def rmsnorm_fixed_order(x, r, w, eps, dtype, w_dtype=None, threads=None):
    """RMSNorm (``r`` None) or fused residual RMSNorm with the CUDA kernels'
    summation order instead of the reference's: a model of the kernels used to
    check them bit for bit. Returns ``y`` or ``(y, residual_out)``."""
    x, w = _c(x), _c(w)
    r = None if r is None else _c(r)
    y = np.empty_like(x)
    ro = np.empty_like(x) if r is not None else None
    h = x.shape[-1]
    rc = lib().ako_oracle_rmsnorm_fixed_order(
        x.ctypes.data, None if r is None else r.ctypes.data, w.ctypes.data, _CODE[w_dtype or dtype], y.ctypes.data,
        None if ro is None else ro.ctypes.data, x.size // h, h, float(eps), _CODE[dtype],
        threads or default_threads())
    if rc != 0:
        raise ValueError(f"rmsnorm_fixed_order: rows of {h} {dtype} elements are not whole 16-byte vectors")
    return y if r is None else (y, ro)


def rope(x, cos, sin, style, dtype, threads=None):
    x = _c(x)
    cos = _c(cos.astype(np.float32))
    sin = _c(sin.astype(np.float32))
    y = np.empty_like(x)
    b, s, h, d = x.shape
    lib().ako_oracle_rope(x.ctypes.data, cos.ctypes.data, sin.ctypes.data, y.ctypes.data, b, s, h, d,
                          1 if style == "interleaved" else 0, _CODE[dtype], threads or default_threads())
    return y


def swiglu(g, u, dtype, threads=None):
    g, u = _c(g), _c(u)
    y = np.empty_like(g)
    h = g.shape[-1] if g.ndim else 1
    lib().ako_oracle_swiglu(g.ctypes.data, u.ctypes.data, y.ctypes.data, g.size // max(h, 1), h, _CODE[dtype],
                            threads or default_threads())
    return y


__all__ = ["build", "lib", "rmsnorm", "rmsnorm_residual", "rmsnorm_fixed_order", "rope", "swiglu", "storage_dtype", "default_threads"]
