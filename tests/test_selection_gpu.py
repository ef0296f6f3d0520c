"""Measured selection on a B200: the validate -> benchmark -> cache loop picks
the sm_100a kernels and records them in ``kernel_cache.json``.

The mirror dispatcher always runs. The reference's own dispatcher runs too
when its package was installed next to the repository (``baseline/_ref``);
RoPE and packed SwiGLU are the ops where ours wins by a wide margin
against AKO's Triton kernels, so the choice is deterministic there.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest
import torch

from ako_b200 import api
from ako_b200.dispatch.cache import KernelCache
from ako_b200.dispatch.hardware import get_device_info
from ako_b200.dispatch.selector import KernelSelector

pytestmark = pytest.mark.gpu

REF_INSTALL = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


def _inputs(dev):
    g = torch.Generator(device=dev).manual_seed(0)
    bf = torch.bfloat16
    x = torch.randn(8192, 4096, device=dev, generator=g).to(bf)
    r = torch.randn(8192, 4096, device=dev, generator=g).to(bf)
    w = (torch.randn(4096, device=dev, generator=g) * 0.1 + 1).to(bf)
    q = torch.randn(8, 512, 32, 128, device=dev, generator=g).to(bf)
    cos, sin = api.build_rope_tables(512, 128, device=dev)
    packed = (torch.randn(2048, 2 * 14336, device=dev, generator=g) * 2).to(bf)
    return x, r, w, q, cos, sin, packed


def test_mirror_selector_picks_the_cuda_kernels(cuda_device, tmp_path) -> None:
    api.register_all(force=True)
    sel = KernelSelector(cache=KernelCache(tmp_path / "kernel_cache.json"), warmup=3, repeats=10)
    x, r, w, q, cos, sin, packed = _inputs(cuda_device)
    calls = [
        ("rmsnorm", (x, w), {}, None),
        ("rmsnorm_residual", (x, r, w), {}, None),
        ("rope", (q, cos, sin), {"style": "neox"}, "neox"),
        ("rope_qk", (q, q[:, :, :8], cos, sin), {"style": "neox"}, "neox"),
        ("swiglu", (packed[:, :14336], packed[:, 14336:]), {}, None),
    ]
    for op, args, kw, extra in calls:
        res = sel.select_entry(op, *args, extra_key=extra, call_kwargs=kw)
        assert res.entry.kernel_name == f"{op}_cuda_sm100", (op, res.to_dict())
        assert not any("cuda_sm100" in rej for rej in res.rejected), res.rejected
        assert res.max_error is not None and res.speedup and res.speedup > 1.0
    doc = json.loads((tmp_path / "kernel_cache.json").read_text())
    gpu_key = get_device_info(cuda_device).cache_key
    assert gpu_key.startswith("NVIDIA_B200")
    recorded = {op: next(iter(shapes.values()))["kernel"] for op, shapes in doc["entries"][gpu_key].items()}
    assert recorded == {op: f"{op}_cuda_sm100" for op, *_ in calls}


def test_reference_selector_picks_the_cuda_kernels(cuda_device, tmp_path, monkeypatch) -> None:
    if not (REF_INSTALL / "ako" / "__init__.py").exists():
        pytest.skip("the reference package is not installed next to the repository")
    monkeypatch.syspath_prepend(str(REF_INSTALL))
    for mod in [m for m in sys.modules if m == "ako" or m.startswith("ako.")]:
        monkeypatch.delitem(sys.modules, mod)
    monkeypatch.setenv("AKO_CACHE_PATH", str(tmp_path / "ako_cache.json"))
    import ako
    from ako.dispatcher.selector import get_selector, reset_selector
    from ako.ops._registry import register_all

    import ako_b200

    reset_selector()
    register_all(force=True)  # AKO's reference, baselines and Triton kernels
    ako_b200.register()  # + the sm_100a candidates, into AKO's registry
    x, r, w, q, cos, sin, packed = _inputs(cuda_device)
    res = get_selector().select_entry("rope", q, cos, sin, extra_key="neox", call_kwargs={"style": "neox"})
    assert res.entry.kernel_name == "rope_cuda_sm100", res.to_dict()
    res = get_selector().select_entry("swiglu", packed[:, :14336], packed[:, 14336:])
    assert res.entry.kernel_name == "swiglu_cuda_sm100", res.to_dict()
    res = get_selector().select_entry("rmsnorm_residual", x, r, w)
    assert not any("cuda_sm100" in rej for rej in res.rejected), res.rejected
    # the public API now runs the selected kernel
    y = ako.rope(q, cos, sin)
    assert torch.equal(y, ako_b200.rope_cuda_sm100(q, cos, sin))
    doc = json.loads((tmp_path / "ako_cache.json").read_text())
    kernels_recorded = {rec["kernel"] for ops in doc["entries"].values() for shapes in ops.values()
                        for rec in shapes.values()}
    assert {"rope_cuda_sm100", "swiglu_cuda_sm100"} <= kernels_recorded
    reset_selector()
