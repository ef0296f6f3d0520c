"""Plain RMSNorm on rows wider than the benchmark's (16385-65536 elements):
the row-resident kernel against the built-in choice, which sends plain 16-bit
rows of 16385-32768 elements (from 1024 rows) to the staged kernel and of
32769-65536 elements (fp16 from 128 rows, bf16 from 1024) to the chunked kernel.

    python -m ako_b200.benchmark.wide_rows            # timing table
    python -m ako_b200.benchmark.wide_rows --capture  # one launch of each wide-row kernel, for ncu

Timing is cold-L2 and differential (ako_b200.benchmark.timing.cold_us); each
line also checks that the two paths give bit-identical outputs. With
``--capture`` each of the two kernels runs once on a case larger than L2,
after a read of twice the L2 size, inside an NVTX range named ``measured``:

    ncu --set full --clock-control none --nvtx --nvtx-include "measured/" \\
        -k regex:"rms_chunk_kernel|rms_tma_kernel" -c 2 -o prof python -m ako_b200.benchmark.wide_rows --capture
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from ako_b200 import _native, kernels
from ako_b200.benchmark.timing import Flusher, cold_us

CELLS = (
    ("bf16", 2048, 32768), ("bf16", 8192, 32768), ("fp16", 16384, 24576), ("bf16", 1024, 32768),
    ("bf16", 148, 65528), ("fp16", 148, 65536), ("bf16", 1024, 65536), ("bf16", 2048, 65536),
    ("bf16", 8192, 65536), ("fp16", 8192, 65536), ("bf16", 8192, 40960), ("fp32", 8192, 32768),
)
DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}


def _peak() -> float:
    try:
        return float(json.loads(Path("MEASURED_PEAKS.json").read_text())["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def _inputs(dt: torch.dtype, rows: int, h: int, dev: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(rows, h, generator=g, device=dev).to(dt)
    w = (torch.randn(h, generator=g, device=dev) * 0.1 + 1).to(dt)
    return x, w


def table() -> None:
    dev = torch.device("cuda", 0)
    lib = _native.lib()
    flush = Flusher(dev)
    peak = _peak()
    print(f"plain rmsnorm, cold L2, fraction of {peak:.1f} GB/s")
    for name, rows, h in CELLS:
        dt = DTYPES[name]
        x, w = _inputs(dt, rows, h, dev)
        nbytes = (2 * rows * h + h) * x.element_size()
        res = {}
        outs = {}
        try:
            for label, mode in (("row-resident", 1), ("built-in", 0)):
                assert lib.ako_b200_rmsnorm_set_staging(mode, 0, 0) == 0
                outs[label] = kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
                res[label] = cold_us(lambda: kernels.rmsnorm_cuda_sm100(x, w, 1e-6), flush, n=6, blocks=3)
        finally:
            lib.ako_b200_rmsnorm_set_staging(0, 0, 0)
        same = torch.equal(outs["row-resident"], outs["built-in"])
        cells = "  ".join(f"{k} {v:8.1f} us ({nbytes / v / 1e3 / peak:.2f})" for k, v in res.items())
        print(f"{name} {rows:5d} x {h:5d}: {cells}  bit-identical={same}", flush=True)
        del x, w, outs
    print("device status", _native.take_device_status())


def capture() -> None:
    dev = torch.device("cuda", 0)
    cases = [("rms_chunk_kernel: rmsnorm bf16 2048 x 65536", *_inputs(torch.bfloat16, 2048, 65536, dev)),
             ("rms_tma_kernel: rmsnorm bf16 4096 x 32768", *_inputs(torch.bfloat16, 4096, 32768, dev))]
    flush = torch.empty(2 * 126 * 2**20 // 8, dtype=torch.int64, device=dev)
    sink = torch.empty((), dtype=torch.int64, device=dev)
    for _, x, w in cases:
        for _ in range(3):
            kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
    for label, x, w in cases:
        torch.sum(flush, dim=0, out=sink)
        torch.cuda.nvtx.range_push("measured")
        kernels.rmsnorm_cuda_sm100(x, w, 1e-6)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        print(f"{label}: {(2 * x.numel() + w.numel()) * x.element_size()} algorithmic bytes", flush=True)
    print("device status", _native.take_device_status())


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--capture", action="store_true")
    args = ap.parse_args()
    capture() if args.capture else table()


if __name__ == "__main__":
    main()
