"""The AKO-facing boundary, on CPU.

* The mirror dispatcher (``ako_b200.dispatch``) follows the selection rule:
  forced, cached, default, validate -> benchmark -> cache; broken or wrong
  candidates are rejected with the reference's messages.
* Where the reference package is importable (its source tree on this
  machine; never on GPU boxes), the mirror is checked against it directly:
  same shape keys, budgets and ulp reports, the same cache file readable by
  both, and ``ako_b200.register()`` plugging the CUDA candidates into the
  reference's own registry, whose selector records them as rejected on CPU
  tensors (no CPU fallback) and keeps its reference.
"""

from __future__ import annotations

import json
import sys
import time

import pytest
import torch

from ako_b200 import api, kernels, plugin
from ako_b200.dispatch import numerical as num
from ako_b200.dispatch import references as refs
from ako_b200.dispatch.cache import CACHE_SCHEMA_VERSION, KernelCache
from ako_b200.dispatch.registry import KernelEntry, KernelRegistry
from ako_b200.dispatch.selector import KernelSelector, SelectionResult, shape_key
from conftest import reference_path


def _selector(tmp_path, *entries, **kw) -> KernelSelector:
    reg = KernelRegistry()
    reg.register(KernelEntry("rmsnorm", "rmsnorm_ref", refs.rmsnorm_ref, "pytorch", 10))
    for e in entries:
        reg.register(e)
    return KernelSelector(registry=reg, cache=KernelCache(tmp_path / "cache.json"), warmup=1, repeats=3,
                          allow_cpu_tuning=True, **kw)


def _slow(x, w, eps=1e-6):
    time.sleep(0.002)
    return refs.rmsnorm_ref(x, w, eps)


def _wrong(x, w, eps=1e-6):
    return torch.zeros_like(x)


def _raises(x, w, eps=1e-6):
    raise RuntimeError("boom")


def test_registry_order_and_replacement() -> None:
    reg = KernelRegistry()
    reg.register(KernelEntry("rmsnorm", "a", _slow, "x", 1))
    reg.register(KernelEntry("rmsnorm", "b", _slow, "x", 5))
    reg.register(KernelEntry("rmsnorm", "c", _slow, "x", 5))
    assert [e.kernel_name for e in reg.list_kernels("rmsnorm")] == ["b", "c", "a"]
    reg.register(KernelEntry("rmsnorm", "b", _wrong, "y", 0))
    assert [e.kernel_name for e in reg.list_kernels("rmsnorm")] == ["c", "a", "b"]
    assert reg.default("rmsnorm").kernel_name == "c" and reg.get("rmsnorm", "b").fn is _wrong
    assert reg.list_ops() == ["rmsnorm"] and reg.default("nope") is None


def test_selector_rejects_wrong_and_raising_and_caches(tmp_path) -> None:
    sel = _selector(tmp_path, KernelEntry("rmsnorm", "wrong", _wrong, "custom", 5),
                    KernelEntry("rmsnorm", "raises", _raises, "custom", 4))
    x, w = torch.randn(64, 512), torch.ones(512)
    res = sel.select_entry("rmsnorm", x, w)
    assert res.entry.kernel_name == "rmsnorm_ref" and res.source == "benchmark"
    reasons = dict(r.split(": ", 1) for r in res.rejected)
    assert "ulps" in reasons["wrong"] and reasons["raises"] == "RuntimeError: boom"
    doc = json.loads((tmp_path / "cache.json").read_text())
    assert doc["version"] == CACHE_SCHEMA_VERSION
    rec = doc["entries"]["cpu_-1"]["rmsnorm"][shape_key((x, w))]
    assert rec["kernel"] == "rmsnorm_ref" and rec["backend"] == "pytorch" and "error_budget" in rec
    again = sel.select_entry("rmsnorm", x, w)
    assert again.source == "cache" and again.from_cache


def test_selector_forced_default_and_memo(tmp_path) -> None:
    sel = _selector(tmp_path, KernelEntry("rmsnorm", "slow", _slow, "custom", 5), auto_tune=False)
    x, w = torch.randn(4, 64), torch.ones(64)
    assert sel.select_entry("rmsnorm", x, w).source == "default"
    assert sel.select_entry("rmsnorm", x, w, forced="slow").source == "forced"
    with pytest.raises(ValueError, match="Unknown kernel 'nope'"):
        sel.select_entry("rmsnorm", x, w, forced="nope")
    fn = sel.select("rmsnorm", x, w)
    assert sel.select("rmsnorm", x, w) is fn and fn is refs.rmsnorm_ref
    with pytest.raises(ValueError, match="No kernels registered"):
        sel.select_entry("swiglu", x, x)


def test_selection_result_record_fields() -> None:
    e = KernelEntry("rmsnorm", "k", _slow, "cuda", 6)
    d = SelectionResult("rmsnorm", e, "key", "benchmark", 0.5, 1.0, 0.0, 2, ("x: y",), 0.75, "rmsnorm_ref").to_dict()
    assert d["speedup"] == 2.0 and d["speedup_vs_best_baseline"] == 1.5 and d["selected_kernel"] == "k"
    assert set(d) == {"operation", "selected_kernel", "backend", "shape_key", "source", "from_cache",
                      "latency_p50_ms", "baseline_ms", "speedup", "best_baseline_ms", "best_baseline_kernel",
                      "speedup_vs_best_baseline", "max_error", "candidates_evaluated", "rejected"}


def test_cache_corrupt_file_and_v1_upgrade(tmp_path) -> None:
    p = tmp_path / "c.json"
    p.write_text("{not json")
    c = KernelCache(p)
    assert len(c) == 0 and (tmp_path / "c.json.corrupt").exists()
    p.write_text(json.dumps({"NVIDIA_B200_0": {"rmsnorm": {"k": "rmsnorm_cuda_sm100"}}}))
    c = KernelCache(p)
    assert c.get("NVIDIA_B200_0", "rmsnorm", "k") == "rmsnorm_cuda_sm100"
    assert c.stats().hits == 1


def test_cache_merges_concurrent_writers(tmp_path) -> None:
    p = tmp_path / "shared.json"
    a, b = KernelCache(p), KernelCache(p)  # two processes' views, loaded before either saved
    a.set("NVIDIA_B200_0", "rmsnorm", "k0", "x")
    b.set("NVIDIA_B200_1", "rmsnorm", "k1", "y")
    merged = KernelCache(p)
    assert merged.get("NVIDIA_B200_0", "rmsnorm", "k0") == "x"
    assert merged.get("NVIDIA_B200_1", "rmsnorm", "k1") == "y"


def test_numerics_gate_values() -> None:
    assert num.ulp(torch.bfloat16, 5.19) == pytest.approx(0.03125)
    assert num.ulp(torch.float16, 5.19) == pytest.approx(2**-8)
    assert num.ulp(torch.float32, 5.19) == pytest.approx(2**-21)
    assert num.ulp(torch.bfloat16, 0.0) > 0
    ref = torch.tensor([4.0, -5.0], dtype=torch.bfloat16)
    assert num.error_budget(ref) == pytest.approx(1e-5 + 1.6e-2 * 5.0)
    assert num.error_budget((ref, ref * 10)) == pytest.approx(1e-5 + 1.6e-2 * 50.0)
    shifted = (ref.float() + 0.03125).to(torch.bfloat16)
    assert num.error_in_ulps(ref, shifted) == pytest.approx(1.0)
    a = torch.tensor([1.0, -1.0, 0.0], dtype=torch.bfloat16)
    b = torch.tensor([1.0 + 2**-7, -1.0 - 2**-7, -0.0], dtype=torch.bfloat16)
    assert num.ulp_distance(a, b).tolist() == [1, 1, 0]


def test_api_dispatch_on_cpu_uses_the_reference_entry() -> None:
    """On CPU the selector does not tune; the reference entry (priority 10)
    runs and the CUDA candidates are registered but not called."""
    api.register_all(force=True)
    x, w = torch.randn(3, 64), torch.randn(64)
    torch.testing.assert_close(api.rmsnorm(x, w), refs.rmsnorm_ref(x, w))
    q = torch.randn(1, 4, 2, 8)
    cos, sin = api.build_rope_tables(4, 8)
    qo, ko = api.rope_qk(q, q, cos, sin)
    torch.testing.assert_close(qo, refs.rope_ref(q, cos, sin))
    with pytest.raises(ValueError, match="requires a CUDA tensor"):
        api.rmsnorm(x, w, kernel="rmsnorm_cuda_sm100")
    names = {e.kernel_name for e in api.get_registry().list_kernels("rmsnorm")}
    assert {"rmsnorm_ref", "rmsnorm_torch_native", "rmsnorm_cuda_sm100"} <= names


# ---------------------------------------------------------- against AKO itself
@pytest.fixture()
def ako_pkg(monkeypatch):
    path = reference_path()
    if path is None:
        pytest.skip("the reference package is not on this machine")
    monkeypatch.syspath_prepend(str(path))
    for mod in [m for m in sys.modules if m == "ako" or m.startswith("ako.")]:
        monkeypatch.delitem(sys.modules, mod)
    import ako
    from ako.dispatcher import selector as ako_selector

    ako_selector.reset_selector()
    yield ako
    ako_selector.reset_selector()
    for mod in [m for m in sys.modules if m == "ako" or m.startswith("ako.")]:
        monkeypatch.delitem(sys.modules, mod)


def test_mirror_matches_reference_keys_budgets_and_records(ako_pkg, tmp_path) -> None:
    from ako.dispatcher.cache import KernelCache as AkoCache
    from ako.dispatcher.selector import shape_key as ako_shape_key
    from ako.validation import numerical as ako_num

    for args in ((torch.randn(2, 3, 64, dtype=torch.bfloat16), torch.ones(64)),
                 (torch.randn(1, 5, 4, 8), torch.ones(5, 4), torch.ones(5, 4))):
        assert shape_key(args) == ako_shape_key(args)
        assert shape_key(args, "neox") == ako_shape_key(args, "neox")
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        ref = (torch.randn(257) * 3).to(dt)
        out = (ref.float() + torch.randn(257) * 0.01).to(dt)
        assert num.error_budget(ref) == ako_num.error_budget(ref)
        assert num.error_in_ulps(ref, out) == ako_num.error_in_ulps(ref, out)
        assert num.ulp(dt, 3.7) == ako_num.ulp(dt, 3.7)
    ours = KernelCache(tmp_path / "k.json")
    ours.set("NVIDIA_B200_0", "rmsnorm", "key", "rmsnorm_cuda_sm100", latency_p50_ms=0.01, backend="cuda")
    theirs = AkoCache(tmp_path / "k.json")
    assert theirs.get_record("NVIDIA_B200_0", "rmsnorm", "key")["kernel"] == "rmsnorm_cuda_sm100"
    theirs.set("NVIDIA_B200_0", "rope", "k2", "rope_cuda_sm100")
    assert KernelCache(tmp_path / "k.json").get("NVIDIA_B200_0", "rope", "k2") == "rope_cuda_sm100"


def test_register_into_the_reference_registry(ako_pkg, tmp_path) -> None:
    """The drop-in: AKO's registry holds the CUDA candidates with AKO's own
    KernelEntry type; AKO's selector, tuning on CPU tensors, records them as
    rejected (ValueError: requires a CUDA tensor) and keeps its reference."""
    from ako.dispatcher.cache import KernelCache as AkoCache
    from ako.dispatcher.registry import KernelEntry as AkoEntry
    from ako.dispatcher.registry import get_registry
    from ako.dispatcher.selector import KernelSelector as AkoSelector
    from ako.ops._registry import register_all

    register_all()
    assert plugin.ako_available()
    reg = plugin.register()
    assert reg is get_registry()
    for op, name, fn in kernels.CANDIDATES:
        entry = reg.get(op, name)
        assert isinstance(entry, AkoEntry) and entry.fn is fn and entry.backend == "cuda" and entry.priority == 6
    assert reg.default("rmsnorm").kernel_name == "rmsnorm_ref"  # the reference stays the default
    sel = AkoSelector(registry=reg, cache=AkoCache(tmp_path / "c.json"), warmup=1, repeats=2,
                      allow_cpu_tuning=True)
    x, w = torch.randn(8, 256), torch.ones(256)
    res = sel.select_entry("rmsnorm", x, w)
    assert any(r.startswith("rmsnorm_cuda_sm100: ValueError") and "requires a CUDA tensor" in r for r in res.rejected)
    assert res.entry.backend in ("pytorch", "torch_native")
    # forced dispatch through the reference's public API reaches our KernelFn
    with pytest.raises(ValueError, match="requires a CUDA tensor"):
        ako_pkg.rmsnorm(x, w, kernel="rmsnorm_cuda_sm100")
    out = ako_pkg.rmsnorm(x, w, kernel="rmsnorm_ref")
    torch.testing.assert_close(out, refs.rmsnorm_ref(x, w))
