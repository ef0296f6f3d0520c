"""Reader for the committed golden vectors (``tests/golden/golden.npz``)."""

from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden.npz"


@lru_cache(maxsize=1)
def load() -> tuple[dict[str, np.ndarray], list[dict]]:
    with np.load(GOLDEN) as z:
        arrays = {k: z[k] for k in z.files}
    cases = json.loads(arrays.pop("cases.json").tobytes().decode())
    return arrays, cases


def cases(op: str | None = None) -> list[dict]:
    _, all_cases = load()
    return [c for c in all_cases if op is None or c["op"] == op]


def arr(case: dict, key: str) -> np.ndarray:
    arrays, _ = load()
    return arrays[f"{case['name']}.{key}"]


def table_rows() -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    arrays, _ = load()
    return arrays["table_8192x128.rows"], arrays["table_8192x128.cos"], arrays["table_8192x128.sin"]
