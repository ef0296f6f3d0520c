"""Measured selection on a B200, through the reference's own dispatcher.

After ``ako_b200.register(b200_timing=True)``, AKO's selector validates and
benchmarks the sm_100a candidates next to AKO's reference, torch baselines
and Triton kernels, with each call timed from a cold L2 (a flush of twice the
B200's 126 MB L2 instead of AKO's stock 32 MiB), and records its decisions in
``kernel_cache.json``. RoPE, packed SwiGLU and the fused q/k RoPE are the ops
where ours wins by a wide margin, so the choice is deterministic there.
"""

from __future__ import annotations

import importlib
import json

import pytest
import torch

import ako_b200
from ako_b200.reference import ako

pytestmark = pytest.mark.gpu


def _inputs(dev):
    g = torch.Generator(device=dev).manual_seed(0)
    bf = torch.bfloat16
    x = torch.randn(8192, 4096, device=dev, generator=g).to(bf)
    r = torch.randn(8192, 4096, device=dev, generator=g).to(bf)
    w = (torch.randn(4096, device=dev, generator=g) * 0.1 + 1).to(bf)
    q = torch.randn(8, 512, 32, 128, device=dev, generator=g).to(bf)
    cos, sin = ako_b200.build_rope_tables(512, 128, device=dev)
    packed = (torch.randn(2048, 2 * 14336, device=dev, generator=g) * 2).to(bf)
    return x, r, w, q, cos, sin, packed


def test_reference_selector_picks_the_cuda_kernels(cuda_device, tmp_path, monkeypatch) -> None:
    pkg = ako()
    monkeypatch.setenv("AKO_CACHE_PATH", str(tmp_path / "ako_cache.json"))
    bench = importlib.import_module("ako.benchmark.bench_op")
    monkeypatch.setattr(bench, "L2_FLUSH_BYTES", bench.L2_FLUSH_BYTES)  # restored after the test
    from ako.dispatcher.hardware import get_device_info
    from ako.dispatcher.selector import get_selector, reset_selector
    from ako.ops._registry import register_all

    reset_selector()
    try:
        register_all(force=True)  # AKO's reference, baselines and Triton kernels
        ako_b200.register(b200_timing=True, shared_cache=True)  # + the sm_100a candidates
        l2 = get_device_info(cuda_device).l2_bytes
        assert l2 and l2 >= 100 << 20
        assert bench.L2_FLUSH_BYTES == 2 * l2
        x, r, w, q, cos, sin, packed = _inputs(cuda_device)
        sel = get_selector()
        res = sel.select_entry("rope", q, cos, sin, extra_key="neox", call_kwargs={"style": "neox"})
        assert res.entry.kernel_name == "rope_cuda_sm100", res.to_dict()
        # the flush AKO's bench_op ran before every timed call was twice the L2
        assert bench._flush_buffer(cuda_device).numel() == 2 * l2
        res = sel.select_entry("swiglu", packed[:, :14336], packed[:, 14336:])
        assert res.entry.kernel_name == "swiglu_cuda_sm100", res.to_dict()
        res = sel.select_entry("rope_qk", q, q[:, :, :8], cos, sin, extra_key="neox", call_kwargs={"style": "neox"})
        assert res.entry.kernel_name == "rope_qk_cuda_sm100", res.to_dict()
        res = sel.select_entry("rmsnorm_residual", x, r, w)
        assert not any("cuda_sm100" in rej for rej in res.rejected), res.rejected
        res = sel.select_entry("rmsnorm", x, w)
        assert not any("cuda_sm100" in rej for rej in res.rejected), res.rejected
        # the public APIs now run the selected kernels
        assert torch.equal(pkg.rope(q, cos, sin), ako_b200.rope_cuda_sm100(q, cos, sin))
        qo, ko = ako_b200.rope_qk(q, q[:, :, :8], cos, sin)
        assert torch.equal(ko, ako_b200.rope_cuda_sm100(q[:, :, :8], cos, sin))
        doc = json.loads((tmp_path / "ako_cache.json").read_text())
        recorded = {rec["kernel"] for ops in doc["entries"].values() for shapes in ops.values()
                    for rec in shapes.values()}
        assert {"rope_cuda_sm100", "swiglu_cuda_sm100", "rope_qk_cuda_sm100"} <= recorded
        gpu_key = get_device_info(cuda_device).cache_key
        assert gpu_key.startswith("NVIDIA_B200")
    finally:
        reset_selector()
        bench._flush_buffer.cache_clear()
        bench._flush_cost_ms.cache_clear()
