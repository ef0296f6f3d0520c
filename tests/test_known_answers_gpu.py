"""The reference's known answers and properties, on the B200 kernels.

AKO's own tests pin its ops with a handful of exact values and invariants
(reference ``tests/test_rmsnorm.py:24-29``, ``tests/test_rmsnorm_residual.py:18-27``,
``tests/test_rope.py:16-84``, ``tests/test_swiglu.py:21-24``): the RMSNorm of
``[3, 4]``, the fused form as a composition, the identity rotation at position
0, norms kept by a rotation, rotated dot products that depend only on the
distance between positions, a table offset equal to later positions, and a
zero ``up`` giving zero. Here each one is checked on the GPU through AKO's
public ops with the sm_100a candidate forced by name (``kernel=``), the way a
user would pin it, so the whole drop-in path (AKO's selector, the KernelFn, the
C ABI, the kernel) is what is tested.
"""

from __future__ import annotations

import math

import pytest
import torch

import ako_b200

pytestmark = pytest.mark.gpu


def test_rmsnorm_of_three_four(cuda_device) -> None:
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        x = torch.tensor([[3.0, 4.0]], device=cuda_device, dtype=dtype)
        w = torch.ones(2, device=cuda_device, dtype=dtype)
        y = ako_b200.rmsnorm(x, w, 1e-6, kernel="rmsnorm_cuda_sm100").float()
        # mean of squares 12.5: y = x / sqrt(12.5 + eps)
        expected = torch.tensor([[3.0, 4.0]], device=cuda_device) / math.sqrt(12.5 + 1e-6)
        tol = 1e-6 if dtype == torch.float32 else (2e-3 if dtype == torch.float16 else 1e-2)
        torch.testing.assert_close(y, expected, atol=tol, rtol=tol)


def test_rmsnorm_residual_is_the_composition(cuda_device) -> None:
    g = torch.Generator(device=cuda_device).manual_seed(3)
    for dtype in (torch.float32, torch.bfloat16):
        x = torch.randn(5, 3, 4096, generator=g, device=cuda_device).to(dtype)
        r = torch.randn(5, 3, 4096, generator=g, device=cuda_device).to(dtype)
        w = (torch.randn(4096, generator=g, device=cuda_device) * 0.1 + 1).to(dtype)
        y, new_r = ako_b200.rmsnorm_residual(x, r, w, 1e-5, kernel="rmsnorm_residual_cuda_sm100")
        assert torch.equal(new_r, x + r)  # the sum rounded once in the storage dtype
        # the normalized part is the plain op on that sum, bit for bit (one summation order per width)
        assert torch.equal(y, ako_b200.rmsnorm(new_r, w, 1e-5, kernel="rmsnorm_cuda_sm100"))


@pytest.mark.parametrize("style", ["neox", "interleaved"])
def test_rope_position_zero_is_the_identity(cuda_device, style: str) -> None:
    x = torch.randn(2, 1, 4, 128, device=cuda_device).to(torch.bfloat16)
    cos, sin = ako_b200.build_rope_tables(8, 128, device=cuda_device)
    y = ako_b200.rope(x, cos[:1], sin[:1], style, kernel="rope_cuda_sm100")
    assert torch.equal(y, x)


@pytest.mark.parametrize("style", ["neox", "interleaved"])
def test_rope_keeps_each_pair_norm(cuda_device, style: str) -> None:
    x = torch.randn(2, 16, 3, 64, device=cuda_device)
    cos, sin = ako_b200.build_rope_tables(16, 64, device=cuda_device)
    y = ako_b200.rope(x, cos, sin, style, kernel="rope_cuda_sm100")
    if style == "neox":
        pairs = lambda t: torch.stack([t[..., :32], t[..., 32:]], -1)  # noqa: E731
    else:
        pairs = lambda t: torch.stack([t[..., 0::2], t[..., 1::2]], -1)  # noqa: E731
    torch.testing.assert_close(pairs(y).norm(dim=-1), pairs(x).norm(dim=-1), atol=1e-5, rtol=1e-5)


def test_rope_dot_products_depend_on_the_distance_only(cuda_device) -> None:
    """q at position m and k at position n: <rope(q)_m, rope(k)_n> depends on
    m - n only, so shifting both positions by the same amount keeps it."""
    head_dim, seq = 64, 32
    q = torch.randn(1, 1, 1, head_dim, device=cuda_device, dtype=torch.float64).float()
    k = torch.randn(1, 1, 1, head_dim, device=cuda_device, dtype=torch.float64).float()
    cos, sin = ako_b200.build_rope_tables(seq, head_dim, device=cuda_device)

    def at(t: torch.Tensor, pos: int) -> torch.Tensor:
        return ako_b200.rope(t, cos[pos:pos + 1], sin[pos:pos + 1], "neox", kernel="rope_cuda_sm100")

    base = (at(q, 7) * at(k, 3)).sum()
    for shift in (1, 5, 20):
        torch.testing.assert_close((at(q, 7 + shift) * at(k, 3 + shift)).sum(), base, atol=1e-4, rtol=1e-4)


def test_rope_table_offset_is_later_positions(cuda_device) -> None:
    """A table built from an offset equals the tail of a longer table, and the
    kernel gives the same bits with either (a decode step at position 2047)."""
    x = torch.randn(3, 1, 8, 128, device=cuda_device).to(torch.bfloat16)
    cos, sin = ako_b200.build_rope_tables(2048, 128, device=cuda_device)
    cos_o, sin_o = ako_b200.build_rope_tables(1, 128, offset=2047, device=cuda_device)
    torch.testing.assert_close(cos_o, cos[2047:], atol=1e-6, rtol=0)
    torch.testing.assert_close(sin_o, sin[2047:], atol=1e-6, rtol=0)
    a = ako_b200.rope(x, cos[2047:], sin[2047:], "neox", kernel="rope_cuda_sm100")
    b = ako_b200.rope(x, cos_o, sin_o, "neox", kernel="rope_cuda_sm100")
    if torch.equal(cos_o, cos[2047:]) and torch.equal(sin_o, sin[2047:]):
        assert torch.equal(a, b)
    else:
        torch.testing.assert_close(a.float(), b.float(), atol=1e-2, rtol=1e-2)


def test_swiglu_zero_up_and_unit_up(cuda_device) -> None:
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        gate = (torch.randn(4, 5632, device=cuda_device) * 2).to(dtype)
        zero = torch.zeros_like(gate)
        y0 = ako_b200.swiglu(gate, zero, kernel="swiglu_cuda_sm100")
        assert not torch.any(y0 != 0)  # silu(g) * 0 is a zero of either sign
        y1 = ako_b200.swiglu(gate, torch.ones_like(gate), kernel="swiglu_cuda_sm100").float()
        g = gate.float()
        tol = 1e-6 if dtype == torch.float32 else (2e-3 if dtype == torch.float16 else 1e-2)
        torch.testing.assert_close(y1, g * torch.sigmoid(g), atol=tol, rtol=tol)
