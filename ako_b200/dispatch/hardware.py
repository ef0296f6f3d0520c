"""Device description and the cache key it contributes.

``DeviceInfo.cache_key`` is ``"<device name with spaces as underscores>_<index>"``
as in the reference (``ako/dispatcher/hardware.py:40-66``), so a B200 record
is keyed ``NVIDIA_B200_<i>`` by either package. Probes are memoized: they sit
on the selection path.
"""

from __future__ import annotations

import shutil
import subprocess
from dataclasses import asdict, dataclass
from functools import lru_cache

import torch


@dataclass(frozen=True)
class DeviceInfo:
    device_type: str
    device_name: str
    device_index: int
    cuda_capability: tuple[int, int] | None
    total_memory_gb: float | None
    driver_version: str | None
    gpu_vendor: str | None = None
    compute_backend: str = "cpu"
    sm_count: int | None = None
    smem_per_block: int | None = None
    l2_bytes: int | None = None
    regs_per_sm: int | None = None

    @property
    def cache_key(self) -> str:
        return f"{self.device_name.replace(' ', '_')}_{self.device_index}"

    def to_dict(self) -> dict:
        return asdict(self)


@lru_cache(maxsize=1)
def _driver_version() -> str | None:
    exe = shutil.which("nvidia-smi")
    if exe is None:
        return None
    try:
        out = subprocess.run([exe, "--query-gpu=driver_version", "--format=csv,noheader"],
                             capture_output=True, text=True, timeout=10, check=True).stdout.strip()
    except (subprocess.SubprocessError, OSError):
        return None
    return out.splitlines()[0].strip() if out else None


@lru_cache(maxsize=None)
def _probe(device_type: str, index: int | None) -> DeviceInfo:
    if device_type == "cuda" and torch.cuda.is_available():
        idx = index if index is not None else torch.cuda.current_device()
        p = torch.cuda.get_device_properties(idx)
        return DeviceInfo(
            device_type="cuda", device_name=p.name, device_index=idx,
            cuda_capability=(p.major, p.minor), total_memory_gb=round(p.total_memory / 2**30, 2),
            driver_version=_driver_version(), gpu_vendor="nvidia", compute_backend="cuda",
            sm_count=p.multi_processor_count,
            smem_per_block=getattr(p, "shared_memory_per_block_optin", None),
            l2_bytes=getattr(p, "L2_cache_size", None),
            regs_per_sm=getattr(p, "regs_per_multiprocessor", None),
        )
    return DeviceInfo(device_type=device_type, device_name="cpu", device_index=-1, cuda_capability=None,
                      total_memory_gb=None, driver_version=None)


def get_device_info(device: torch.device | str | None = None) -> DeviceInfo:
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    elif isinstance(device, str):
        device = torch.device(device)
    return _probe(device.type, device.index)


def clear_device_cache() -> None:
    _probe.cache_clear()
    _driver_version.cache_clear()
