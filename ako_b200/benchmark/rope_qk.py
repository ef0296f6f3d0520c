"""Fused q/k RoPE against two RoPE calls (the reference's ``rope_qk``,
``ako/ops/rope.py:45-58``, which calls ``rope`` for q and then for k).

    python -m ako_b200.benchmark.rope_qk [--out FILE]

q has 32 heads and k 8, head size 128, neox, bf16. Throughput cells are timed
cold-L2 and differentially (ako_b200.benchmark.timing.cold_us) for the pair of
calls and for the fused call; decode cells (one position per sequence) are
timed as device time per pair inside a CUDA graph of 20 pairs, and per pair
of 50 issued back to back from Python (bound by the host's launch rate at
these sizes). Each line checks that both give the same bytes.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from ako_b200 import _native, kernels
from ako_b200.benchmark.sweep import graph_us
from ako_b200.benchmark.timing import Flusher, back_to_back_us, cold_us
from ako_b200.dispatch import references as refs

HQ, HK, D = 32, 8, 128


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    flush = Flusher(dev)
    cos_all, sin_all = refs.build_rope_tables(8192, D, device=dev)
    out = []

    def pair(q, k, cos, sin):
        return kernels.rope_cuda_sm100(q, cos, sin, "neox"), kernels.rope_cuda_sm100(k, cos, sin, "neox")

    def fused(q, k, cos, sin):
        return kernels.rope_qk_cuda_sm100(q, k, cos, sin, "neox")

    for b, s in ((8, 2048), (32, 4096)):
        q = torch.randn(b, s, HQ, D, generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn(b, s, HK, D, generator=g, device=dev).to(torch.bfloat16)
        cos, sin = cos_all[:s], sin_all[:s]
        same = all(torch.equal(x, y) for x, y in zip(pair(q, k, cos, sin), fused(q, k, cos, sin)))
        t2 = cold_us(lambda: pair(q, k, cos, sin), flush, n=6, blocks=3)
        t1 = cold_us(lambda: fused(q, k, cos, sin), flush, n=6, blocks=3)
        nbytes = 2 * (q.numel() + k.numel()) * 2 + s * (D // 2) * 4 * 2
        rec = {"cell": f"B{b} S{s}", "two_calls_us": round(t2, 2), "fused_us": round(t1, 2),
               "fused_gbs": round(nbytes / t1 / 1e3, 1), "identical": same}
        out.append(rec)
        print(rec, flush=True)
        del q, k

    for b in (1, 8, 32):
        q = torch.randn(b, 1, HQ, D, generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn(b, 1, HK, D, generator=g, device=dev).to(torch.bfloat16)
        cos, sin = cos_all[2047:2048], sin_all[2047:2048]
        same = all(torch.equal(x, y) for x, y in zip(pair(q, k, cos, sin), fused(q, k, cos, sin)))
        rec = {"cell": f"decode B{b}", "identical": same,
               "graph_two_calls_us": graph_us(pair, (q, k, cos, sin)), "graph_fused_us": graph_us(fused, (q, k, cos, sin)),
               "wall_two_calls_us": round(back_to_back_us(lambda: pair(q, k, cos, sin)), 2),
               "wall_fused_us": round(back_to_back_us(lambda: fused(q, k, cos, sin)), 2)}
        out.append(rec)
        print(rec, flush=True)
    print("device status", _native.take_device_status())
    if args.out:
        Path(args.out).write_text(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
