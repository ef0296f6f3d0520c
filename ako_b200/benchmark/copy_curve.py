"""Device-to-device copy bandwidth against the bytes moved, timed like the
sweep (cold L2, differential; see ako_b200.benchmark.timing): the practical
roofline for a memory-bound call of a given size, since ramp-up, tail and
launch weigh more the smaller the transfer.

    python -m ako_b200.benchmark.copy_curve [--out copy_curve.json]

Each line is one ``torch.Tensor.copy_`` of half the stated bytes (read plus
write = the stated bytes), with the fraction of the measured copy bandwidth.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from ako_b200.benchmark.timing import Flusher, cold_us

SIZES_MB = (4, 8, 16, 33, 67, 134, 268, 537, 1074, 2148)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", default=None)
    ap.add_argument("--peak-gbs", type=float, default=None)
    args = ap.parse_args()
    peak = args.peak_gbs
    if peak is None:
        try:
            peak = float(json.loads(Path("MEASURED_PEAKS.json").read_text())["hbm_gbs"])
        except (OSError, KeyError, ValueError):
            peak = 6650.0
    dev = torch.device("cuda", 0)
    flush = Flusher(dev)
    out = []
    for mb in SIZES_MB:
        n = mb * 1000 * 1000 // 2
        a = torch.empty(n, dtype=torch.uint8, device=dev)
        b = torch.empty_like(a)
        us = cold_us(lambda: b.copy_(a), flush, n=10 if mb < 500 else 4, blocks=5)
        gbs = 2 * n / us / 1e3
        out.append({"bytes": 2 * n, "us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 3)})
        print(f"copy moving {mb:5d} MB: {us:8.2f} us  {gbs:7.0f} GB/s  {gbs / peak:.3f}", flush=True)
        del a, b
    if args.out:
        Path(args.out).write_text(json.dumps({"peak_gbs": peak, "points": out}, indent=1))


if __name__ == "__main__":
    main()
