"""Generate the golden vectors in this folder from the reference implementation.

Runs AKO's own unfused PyTorch references (``ako.ops.rmsnorm_ref``,
``rope_ref``, ``swiglu_ref``) on CPU over seeded inputs and stores inputs and
outputs as raw storage bits in ``golden.npz`` (bfloat16 as ``uint16``).

It needs the reference source tree importable (``--reference PATH``, default
the ``AKO_REFERENCE`` environment variable); it is run by hand when the cases
change, never by the tests, which only read the committed ``golden.npz``.

    python tests/golden/make_golden.py --reference /path/to/AKO
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "golden.npz"

_TORCH = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def normal(gen: torch.Generator, shape, mean: float, std: float, dtype: str) -> torch.Tensor:
    """N(mean, std) drawn in fp32 on CPU, then cast to the storage dtype."""
    return (torch.randn(*shape, generator=gen, dtype=torch.float32) * std + mean).to(_TORCH[dtype])


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("AKO_REFERENCE"), help="AKO source tree")
    args = ap.parse_args()
    if not args.reference:
        sys.exit("pass --reference or set AKO_REFERENCE")
    sys.path.insert(0, str(Path(args.reference).resolve()))
    from ako.ops.rmsnorm_ref import rmsnorm_ref, rmsnorm_residual_ref
    from ako.ops.rope_ref import build_rope_tables, rope_ref
    from ako.ops.swiglu_ref import swiglu_ref

    arrays: dict[str, np.ndarray] = {}
    cases: list[dict] = []

    def add(name: str, op: str, meta: dict, tensors: dict[str, torch.Tensor]) -> None:
        for k, v in tensors.items():
            arrays[f"{name}.{k}"] = bits(v)
        cases.append({"name": name, "op": op, **meta})

    seed = 0
    # Known answer from the reference's tests: [[3, 4]] -> x / sqrt(12.5).
    x = torch.tensor([[3.0, 4.0]])
    w = torch.ones(2)
    add("rms_known", "rmsnorm", {"dtype": "float32", "eps": 1e-6},
        {"x": x, "w": w, "y": rmsnorm_ref(x, w, 1e-6)})

    for dtype in ("float32", "float16", "bfloat16"):
        for rows, h, eps in ((2, 4096, 1e-6), (3, 100, 1e-5), (1, 8448, 1e-5), (3, 2048, 1e-5)):
            seed += 1
            g = torch.Generator().manual_seed(seed)
            x = normal(g, (rows, h), 0.0, 1.0, dtype)
            w = normal(g, (h,), 1.0, 0.1, dtype)
            add(f"rms_{dtype}_{rows}x{h}", "rmsnorm", {"dtype": dtype, "eps": eps},
                {"x": x, "w": w, "y": rmsnorm_ref(x, w, eps)})
            seed += 1
            g = torch.Generator().manual_seed(seed)
            x = normal(g, (rows, h), 0.0, 1.0, dtype)
            r = normal(g, (rows, h), 0.0, 1.0, dtype)
            w = normal(g, (h,), 1.0, 0.1, dtype)
            y, ro = rmsnorm_residual_ref(x, r, w, eps)
            add(f"res_{dtype}_{rows}x{h}", "rmsnorm_residual", {"dtype": dtype, "eps": eps},
                {"x": x, "r": r, "w": w, "y": y, "ro": ro})

    # RoPE tables: spot rows of the (8192, 128) table the decode config slices.
    cos_full, sin_full = build_rope_tables(8192, 128)
    rows_idx = torch.tensor([0, 1, 2, 1000, 2047, 4095, 8191])
    arrays["table_8192x128.rows"] = rows_idx.numpy()
    arrays["table_8192x128.cos"] = bits(cos_full[rows_idx])
    arrays["table_8192x128.sin"] = bits(sin_full[rows_idx])

    for dtype in ("float32", "float16", "bfloat16"):
        for style in ("neox", "interleaved"):
            for (b, s, hh, d, offset) in ((2, 6, 3, 8, 0), (1, 4, 4, 128, 2044), (2, 3, 8, 128, 0)):
                seed += 1
                g = torch.Generator().manual_seed(seed)
                x = normal(g, (b, s, hh, d), 0.0, 1.0, dtype)
                cos, sin = build_rope_tables(s, d, offset=offset)
                add(f"rope_{dtype}_{style}_{b}x{s}x{hh}x{d}_off{offset}", "rope",
                    {"dtype": dtype, "style": style, "offset": offset},
                    {"x": x, "cos": cos, "sin": sin, "y": rope_ref(x, cos, sin, style)})

    for dtype in ("float32", "float16", "bfloat16"):
        for rows, f in ((2, 5632), (2, 100), (1, 8448)):
            seed += 1
            g = torch.Generator().manual_seed(seed)
            gate = normal(g, (rows, f), 0.0, 2.0, dtype)
            up = normal(g, (rows, f), 0.0, 2.0, dtype)
            add(f"swiglu_{dtype}_{rows}x{f}", "swiglu", {"dtype": dtype},
                {"g": gate, "u": up, "y": swiglu_ref(gate, up)})

    arrays["cases.json"] = np.frombuffer(json.dumps(cases).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(cases)} cases, torch {torch.__version__})")


if __name__ == "__main__":
    main()
