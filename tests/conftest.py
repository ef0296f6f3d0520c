"""Shared fixtures: markers, repository path, isolated kernel cache, GPU gating."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(autouse=True, scope="session")
def isolated_kernel_cache(tmp_path_factory: pytest.TempPathFactory):
    """Keep the suite away from the user's ``~/.ako/kernel_cache.json``."""
    cache_dir = tmp_path_factory.mktemp("ako-cache")
    with pytest.MonkeyPatch.context() as mp:
        mp.setenv("AKO_CACHE_PATH", str(cache_dir / "kernel_cache.json"))
        yield


@pytest.fixture(scope="session")
def cuda_device():
    """The GPU the `gpu` tests run on; fails (does not skip) when there is none."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test needs a CUDA device")
    return torch.device("cuda", 0)


def reference_path() -> Path | None:
    """Directory holding the reference's ``ako`` package (``AKO_REFERENCE``,
    else the offline install under ``baseline/_ref``), when there is one;
    only CPU tests use it."""
    cand = os.environ.get("AKO_REFERENCE")
    p = Path(cand) if cand else Path(__file__).resolve().parents[1] / "baseline" / "_ref"
    return p if (p / "ako" / "__init__.py").exists() else None
