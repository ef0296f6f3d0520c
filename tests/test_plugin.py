"""The drop-in boundary on CPU, against the reference's own dispatcher.

* ``ako_b200.register()`` puts the CUDA candidates into AKO's registry with
  AKO's ``KernelEntry`` type (backend ``cuda``, priority 6), keeps AKO's
  reference the unmeasured default, and adds the ``rope_qk`` op with AKO's
  pair of ``rope_ref`` calls as its baseline.
* AKO's selector, tuning on CPU tensors, records the candidates as rejected
  (``ValueError: requires a CUDA tensor``: there is no CPU fallback).
* ``ako_b200``'s op API is AKO's API: on CPU it returns AKO's reference.
* The two opt-ins: the B200-sized L2 flush of AKO's ``bench_op``, and a
  cache file that several processes can share without losing records.
"""

from __future__ import annotations

import json
import multiprocessing as mp
from pathlib import Path

import pytest
import torch

import ako_b200
from ako_b200 import api, kernels, plugin
from ako_b200.reference import ako, ops


@pytest.fixture()
def fresh_selector():
    ako()
    from ako.dispatcher.selector import reset_selector

    reset_selector()
    yield
    reset_selector()


def test_reference_package_is_the_dependency() -> None:
    pkg = ako()
    assert pkg.__version__ == "0.2.0"
    assert ops().rmsnorm_ref.__module__ == "ako.ops.rmsnorm_ref"


def test_register_into_the_reference_registry(fresh_selector, tmp_path) -> None:
    from ako.dispatcher.cache import KernelCache
    from ako.dispatcher.registry import KernelEntry, get_registry
    from ako.dispatcher.selector import KernelSelector
    from ako.ops._registry import register_all

    register_all()
    reg = ako_b200.register()
    assert reg is get_registry()
    for op, name, fn in kernels.CANDIDATES:
        entry = reg.get(op, name)
        assert isinstance(entry, KernelEntry) and entry.fn is fn and entry.backend == "cuda" and entry.priority == 6
    assert reg.default("rmsnorm").kernel_name == "rmsnorm_ref"  # the reference stays the default
    assert reg.default("rope_qk").kernel_name == "rope_qk_ref" and reg.default("rope_qk").backend == "pytorch"
    sel = KernelSelector(registry=reg, cache=KernelCache(tmp_path / "c.json"), warmup=1, repeats=2,
                         allow_cpu_tuning=True)
    x, w = torch.randn(8, 256), torch.ones(256)
    res = sel.select_entry("rmsnorm", x, w)
    assert any(r.startswith("rmsnorm_cuda_sm100: ValueError") and "requires a CUDA tensor" in r for r in res.rejected)
    assert res.entry.backend in ("pytorch", "torch_native")
    rec = json.loads((tmp_path / "c.json").read_text())["entries"]
    assert rec and all(r["kernel"] != "rmsnorm_cuda_sm100" for ops_ in rec.values() for s in ops_.values()
                       for r in s.values())


def test_op_api_is_akos_api_on_cpu(fresh_selector) -> None:
    """On CPU AKO does not tune: every op returns AKO's reference, a forced CUDA
    candidate raises, and ``rope_qk`` is dispatched as its own op."""
    pkg = ako()
    x, w = torch.randn(3, 64), torch.randn(64)
    torch.testing.assert_close(ako_b200.rmsnorm(x, w), ops().rmsnorm_ref(x, w))
    r = torch.randn(3, 64)
    y, ro = ako_b200.rmsnorm_residual(x, r, w)
    y_ref, ro_ref = ops().rmsnorm_residual_ref(x, r, w)
    assert torch.equal(y, y_ref) and torch.equal(ro, ro_ref)
    g, u = torch.randn(2, 32), torch.randn(2, 32)
    assert torch.equal(ako_b200.swiglu(g, u), ops().swiglu_ref(g, u))
    q, k = torch.randn(1, 4, 2, 8), torch.randn(1, 4, 1, 8)
    cos, sin = api.build_rope_tables(4, 8)
    c2, s2 = pkg.build_rope_tables(4, 8)
    assert torch.equal(cos, c2) and torch.equal(sin, s2)
    assert torch.equal(ako_b200.rope(q, cos, sin), ops().rope_ref(q, cos, sin))
    qo, ko = ako_b200.rope_qk(q, k, cos, sin)
    assert torch.equal(qo, ops().rope_ref(q, cos, sin)) and torch.equal(ko, ops().rope_ref(k, cos, sin))
    qo, ko = ako_b200.rope_qk(q, k, cos, sin, kernel="rope_ref")  # a rope kernel: AKO's two dispatched calls
    assert torch.equal(ko, ops().rope_ref(k, cos, sin))
    with pytest.raises(ValueError, match="requires a CUDA tensor"):
        ako_b200.rmsnorm(x, w, kernel="rmsnorm_cuda_sm100")
    with pytest.raises(ValueError, match="requires a CUDA tensor"):
        ako_b200.rope_qk(q, k, cos, sin, kernel="rope_qk_cuda_sm100")
    # forced dispatch through the reference's own public API reaches our KernelFn
    with pytest.raises(ValueError, match="requires a CUDA tensor"):
        pkg.rope(q, cos, sin, kernel="rope_cuda_sm100")


def test_b200_flush_sizes_akos_bench_op(fresh_selector, monkeypatch) -> None:
    """``register(b200_timing=True)`` sizes AKO's per-call L2 flush to twice the
    device's L2 and drops the cached flush buffer and its calibrated cost."""
    import importlib

    ako()
    ako_bench = importlib.import_module("ako.benchmark.bench_op")
    from ako.dispatcher import hardware

    class Info:
        l2_bytes = 132_120_576  # B200: 126 MiB

    monkeypatch.setattr(hardware, "get_device_info", lambda device=None: Info())
    monkeypatch.setattr(ako_bench, "L2_FLUSH_BYTES", ako_bench.L2_FLUSH_BYTES)
    ako_bench._flush_buffer.cache_clear()
    ako_bench._flush_buffer(torch.device("cpu"))  # a cached buffer of the old size
    assert ako_bench._flush_buffer.cache_info().currsize == 1
    ako_b200.register(b200_timing=True)
    assert ako_bench.L2_FLUSH_BYTES == 2 * Info.l2_bytes
    assert ako_bench._flush_buffer.cache_info().currsize == 0
    assert ako_bench._flush_buffer(torch.device("cpu")).numel() == 2 * Info.l2_bytes
    ako_bench._flush_buffer.cache_clear()


def _writer(path: str, tag: int, n: int, start, locked: bool) -> None:
    from ako_b200.reference import ako

    ako()
    if locked:
        from ako_b200.shared_cache import LockedKernelCache as Cache
    else:
        from ako.dispatcher.cache import KernelCache as Cache
    cache = Cache(Path(path))  # both processes load before either writes
    start.wait()
    for i in range(n):
        cache.set(f"NVIDIA_B200_{tag}", "rmsnorm", f"({i},)_bfloat16", "rmsnorm_cuda_sm100", latency_p50_ms=0.01)


@pytest.mark.parametrize("locked", [True, False], ids=["locked", "ako"])
def test_two_processes_share_one_cache_file(tmp_path, locked: bool) -> None:
    """Two processes that loaded the same file write 40 records each. With the
    locked cache all 80 survive; AKO's own save keeps only what the last
    writer had in memory (the reason for the opt-in)."""
    path = tmp_path / "kernel_cache.json"
    ctx = mp.get_context("spawn")
    start = ctx.Barrier(2)
    procs = [ctx.Process(target=_writer, args=(str(path), t, 40, start, locked)) for t in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    doc = json.loads(path.read_text())
    n = sum(len(s) for ops_ in doc["entries"].values() for s in ops_.values())
    if locked:
        assert n == 80 and doc["version"] == 2
        ako()
        from ako.dispatcher.cache import KernelCache

        assert KernelCache(path).get("NVIDIA_B200_1", "rmsnorm", "(39,)_bfloat16") == "rmsnorm_cuda_sm100"
    else:
        assert n < 80


def test_shared_cache_opt_in_replaces_the_selectors_cache(fresh_selector, tmp_path, monkeypatch) -> None:
    from ako.dispatcher.selector import get_selector

    from ako_b200.shared_cache import LockedKernelCache

    monkeypatch.setenv("AKO_CACHE_PATH", str(tmp_path / "k.json"))
    ako_b200.register(shared_cache=True)
    cache = get_selector().cache
    assert isinstance(cache, LockedKernelCache) and cache.path == tmp_path / "k.json"
    ako_b200.register(shared_cache=True)
    assert get_selector().cache is cache
    cache.set("g", "op", "k", "kern")
    cache.clear()
    assert json.loads((tmp_path / "k.json").read_text())["entries"] == {}


def test_plugin_module_has_no_reference_code_of_its_own() -> None:
    """The package reuses AKO's dispatcher: no selector, cache or numerics of its own."""
    root = Path(ako_b200.__file__).resolve().parent
    assert not (root / "dispatch").exists()
    assert plugin.CUDA_PRIORITY == 6 and plugin.REFERENCE_PRIORITY == 10
