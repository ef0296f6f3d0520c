"""Runs one config cell with the sm_100a kernel and with a competitor, for
side-by-side profiling (``ncu -k regex:...``) of the two kernels.

    python -m ako_b200.benchmark.compare_cell --op rmsnorm --rows 2048 --hidden 4096 --dtype fp32

The competitor is the reference's Triton kernel when the reference package
is importable (``--reference-path``), else ``torch.compile`` of the unfused
reference. Each is launched ``--launches`` times after three warm-up calls,
with a 2 x L2 read between launches so every launch starts with a cold L2;
the measured launches sit in an NVTX range named ``measured``:

    ncu --set full --clock-control none --nvtx --nvtx-include "measured/" \
        -k regex:"rms_rows_kernel|_rmsnorm_kernel_impl" -c 2 -o prof \
        python -m ako_b200.benchmark.compare_cell --op rmsnorm --rows 2048 --hidden 4096 --dtype fp32 --launches 1
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

from ako_b200 import kernels
from ako_b200.dispatch import references as refs

DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--op", choices=("rmsnorm", "rmsnorm_residual", "swiglu"), default="rmsnorm")
    ap.add_argument("--rows", type=int, default=2048)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--dtype", choices=sorted(DTYPES), default="fp32")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--reference-path", default="baseline/_ref")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    dt = DTYPES[args.dtype]
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(args.rows, args.hidden, device=dev, generator=g).to(dt)
    r = torch.randn(args.rows, args.hidden, device=dev, generator=g).to(dt)
    w = (torch.randn(args.hidden, device=dev, generator=g) * 0.1 + 1).to(dt)
    if args.reference_path and Path(args.reference_path).exists():
        sys.path.insert(0, args.reference_path)
    try:
        from ako.ops import rmsnorm_triton, swiglu_triton

        comp = {"rmsnorm": lambda: rmsnorm_triton.rmsnorm_triton(x, w, 1e-6),
                "rmsnorm_residual": lambda: rmsnorm_triton.rmsnorm_residual_triton(x, r, w, 1e-5),
                "swiglu": lambda: swiglu_triton.swiglu_triton(x, r)}[args.op]
    except ImportError:
        comp = {"rmsnorm": lambda: refs.rmsnorm_compiled(x, w, 1e-6),
                "rmsnorm_residual": lambda: refs.rmsnorm_residual_compiled(x, r, w, 1e-5),
                "swiglu": lambda: refs.swiglu_compiled(x, r)}[args.op]
    ours = {"rmsnorm": lambda: kernels.rmsnorm_cuda_sm100(x, w, 1e-6),
            "rmsnorm_residual": lambda: kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5),
            "swiglu": lambda: kernels.swiglu_cuda_sm100(x, r)}[args.op]
    flush = torch.empty(2 * 126 * 2**20, dtype=torch.uint8, device=dev)
    sink = torch.empty((), dtype=torch.int64, device=dev)
    for fn in (ours, comp):  # warm-up (and the competitor's autotuning) first
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("measured")  # ncu --nvtx --nvtx-include "measured/" selects these launches
    for fn in (ours, comp):
        for _ in range(args.launches):
            torch.sum(flush.view(torch.int64), dim=0, out=sink)
            fn()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
