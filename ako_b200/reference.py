"""The reference package (Farx1/AKO, ``import ako``): a declared dependency.

The sm_100a kernels are candidates in AKO's own dispatcher, so ``ako`` must
be importable. It is found, in order:

1. as an installed package (``pip install`` of the reference);
2. under ``AKO_REFERENCE_PATH`` (a directory that contains ``ako/``);
3. under ``baseline/_ref`` next to this package, the offline install a
   source checkout of this repository carries.

:func:`ako` raises :class:`ImportError` naming all three when none has it.
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path
from types import ModuleType

_REPO_INSTALL = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


def _candidates() -> list[Path]:
    out = []
    env = os.environ.get("AKO_REFERENCE_PATH")
    if env:
        out.append(Path(env))
    out.append(_REPO_INSTALL)
    return out


def ako() -> ModuleType:
    """Import and return the reference package ``ako``."""
    try:
        return importlib.import_module("ako")
    except ImportError:
        pass
    for path in _candidates():
        if (path / "ako" / "__init__.py").exists():
            if str(path) not in sys.path:
                sys.path.append(str(path))
            return importlib.import_module("ako")
    raise ImportError(
        "ako_b200 needs the reference package `ako` (Farx1/AKO): install it, or point AKO_REFERENCE_PATH at a "
        f"directory containing ako/ (looked in: {', '.join(str(p) for p in _candidates())})"
    )


def available() -> bool:
    try:
        ako()
    except ImportError:
        return False
    return True


def ops():
    """AKO's unfused reference ops and its RoPE table builder, as one namespace:
    ``rmsnorm_ref``, ``rmsnorm_residual_ref`` (``ako/ops/rmsnorm_ref.py``),
    ``rope_ref``, ``build_rope_tables`` (``ako/ops/rope_ref.py``) and
    ``swiglu_ref`` (``ako/ops/swiglu_ref.py``)."""
    global _OPS
    if _OPS is None:
        ako()
        from types import SimpleNamespace

        from ako.ops.rmsnorm_ref import rmsnorm_ref, rmsnorm_residual_ref
        from ako.ops.rope_ref import build_rope_tables, rope_ref
        from ako.ops.swiglu_ref import swiglu_ref

        _OPS = SimpleNamespace(rmsnorm_ref=rmsnorm_ref, rmsnorm_residual_ref=rmsnorm_residual_ref, rope_ref=rope_ref,
                               build_rope_tables=build_rope_tables, swiglu_ref=swiglu_ref)
    return _OPS


_OPS = None
