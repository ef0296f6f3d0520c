"""Runs the kernels the launch tables do not pick for the benchmark cells, for
ncu captures: the any-width RMSNorm kernel (a ragged row), the vector RoPE
kernel with 4-byte accesses (a head size whose half is an even number of
elements but not of 16-byte vectors), the scalar RoPE kernel (an odd half
head size) and the staged (bulk-copy ring) RMSNorm kernel, which only a
measurement switch selects. Each launch follows a read of twice the L2 size, inside an NVTX
range named ``measured``:

    ncu --set full --clock-control none --nvtx --nvtx-include "measured/" \\
        -k regex:"rms_generic_kernel|rope_scalar_kernel|rope_vec_kernel|rms_tma_kernel" -c 4 -o prof \\
        python -m ako_b200.benchmark.fallbacks

Prints each case's algorithmic bytes, so a capture's durations convert to
achieved GB/s.
"""

from __future__ import annotations

import torch

from ako_b200 import _native, kernels
from ako_b200.dispatch import references as refs


def main() -> None:
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    bf = torch.bfloat16
    rnd = lambda *s: torch.randn(*s, generator=g, device=dev).to(bf)  # noqa: E731
    lib = _native.lib()

    x, r = rnd(8192, 4100), rnd(8192, 4100)
    w = (torch.randn(4100, generator=g, device=dev) * 0.1 + 1).to(bf)
    q = rnd(8, 512, 32, 100)
    cos, sin = refs.build_rope_tables(512, 100, device=dev)
    q98 = rnd(8, 512, 32, 98)
    cos98, sin98 = refs.build_rope_tables(512, 98, device=dev)
    xs, rs = rnd(8192, 4096), rnd(8192, 4096)
    ws = (torch.randn(4096, generator=g, device=dev) * 0.1 + 1).to(bf)

    def staged():
        lib.ako_b200_rmsnorm_set_staging(2, 4, 2)
        try:
            return kernels.rmsnorm_residual_cuda_sm100(xs, rs, ws, 1e-5)
        finally:
            lib.ako_b200_rmsnorm_set_staging(0, 0, 0)

    cases = [
        ("rms_generic_kernel: rmsnorm_residual bf16 8192 x 4100", lambda: kernels.rmsnorm_residual_cuda_sm100(x, r, w, 1e-5),
         (4 * x.numel() + w.numel()) * 2),
        ("rope_vec_kernel, 4-byte accesses: rope neox bf16 8 x 512 x 32 x 100",
         lambda: kernels.rope_cuda_sm100(q, cos, sin, "neox"), 2 * q.numel() * 2 + 512 * 50 * 4 * 2),
        ("rope_scalar_kernel: rope neox bf16 8 x 512 x 32 x 98", lambda: kernels.rope_cuda_sm100(q98, cos98, sin98, "neox"),
         2 * q98.numel() * 2 + 512 * 49 * 4 * 2),
        ("rms_tma_kernel: rmsnorm_residual bf16 8192 x 4096, staged", staged, (4 * xs.numel() + ws.numel()) * 2),
    ]
    flush = torch.empty(2 * 126 * 2**20 // 8, dtype=torch.int64, device=dev)
    sink = torch.empty((), dtype=torch.int64, device=dev)
    for _, fn, _ in cases:
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("measured")
    for _, fn, _ in cases:
        torch.sum(flush, dim=0, out=sink)
        fn()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    status = _native.take_device_status()
    for name, _, nbytes in cases:
        print(f"{name}: {nbytes} algorithmic bytes")
    print(f"device status {status}")
    if status != 0:
        raise SystemExit("a staged kernel's bounded wait ran out")


if __name__ == "__main__":
    main()
