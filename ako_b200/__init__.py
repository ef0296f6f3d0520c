"""B200 (sm_100a) kernels for AKO's memory-bound inference ops.

* :mod:`ako_b200.kernels` — the CUDA candidates with AKO's KernelFn signatures
  (``rmsnorm_cuda_sm100`` …), over the C ABI in ``include/ako_b200.h``.
* :func:`ako_b200.register` — adds them to AKO's dispatcher (drop-in).
* :mod:`ako_b200.api` — AKO's public op API on the package's own dispatcher.
* :mod:`ako_b200.host` — host-buffer entry points (PCIe-pipelined).
* :mod:`ako_b200.bandwidth` — GB/s columns for AKO's benchmark reports.
"""

from ako_b200 import bandwidth
from ako_b200.api import build_rope_tables, rmsnorm, rmsnorm_residual, rope, rope_qk, swiglu
from ako_b200.kernels import (
    rmsnorm_cuda_sm100,
    rmsnorm_residual_cuda_sm100,
    rope_cuda_sm100,
    rope_qk_cuda_sm100,
    swiglu_cuda_sm100,
)
from ako_b200.plugin import register

__version__ = "0.1.0"

__all__ = [
    "__version__",
    "bandwidth",
    "build_rope_tables",
    "register",
    "rmsnorm",
    "rmsnorm_cuda_sm100",
    "rmsnorm_residual",
    "rmsnorm_residual_cuda_sm100",
    "rope",
    "rope_cuda_sm100",
    "rope_qk",
    "rope_qk_cuda_sm100",
    "swiglu",
    "swiglu_cuda_sm100",
]
