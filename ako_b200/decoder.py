"""LLaMA-style decoder with RMSNorm, RoPE and SwiGLU on the sm_100a kernels.

The caller of the hot path that benchmark configuration 5 measures (reference:
``ako/models/decoder.py:37-335``): a stack of pre-norm blocks —
``norm -> attention -> norm -> SwiGLU MLP`` with the residual carried through
the fused residual-add RMSNorm — plus the token embedding and LM head the
reference's stack leaves to its harness. Same configuration fields and
norm/residual order as the reference; the layout is chosen for B200:

* q, k and v come out of one packed GEMM and stay views of it; the fused
  ``rope_qk`` kernel reads q and k in place and writes the rotated keys
  straight into the KV cache (output strides are free in the C ABI);
* gate and up come out of one packed GEMM; the SwiGLU kernel reads the two
  halves in place;
* the KV cache is preallocated ``(batch, kv_heads, max_len, head_dim)`` per
  layer and written in place, where the reference concatenates the whole
  cache every step (``ako/models/decoder.py:84-93``);
* grouped-query attention goes through SDPA with ``enable_gqa`` instead of
  materializing repeated heads (``ako/models/decoder.py:180-182``).

GEMMs and attention are torch's (cuBLAS / SDPA), as config 5 specifies.
``backend="torch"`` runs the same stack with the unfused reference math for
RMSNorm, RoPE and SwiGLU (AKO's own ``ako.ops.*_ref``), for comparison.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch
import torch.nn.functional as F
from torch import nn

from ako_b200 import _native, kernels
from ako_b200.reference import ops as reference_ops

Backend = Literal["b200", "torch"]


@dataclass
class ModelConfig:
    """Shape of the stack (fields of the reference's ``ModelConfig``, plus vocab)."""

    hidden_dim: int = 4096
    n_layers: int = 4
    n_heads: int = 32
    n_kv_heads: int = 8
    intermediate_dim: int = 11008
    max_seq_len: int = 8192
    rope_base: float = 10000.0
    rope_style: str = "neox"
    eps: float = 1e-5
    vocab_size: int = 32000

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.n_heads

    def __post_init__(self) -> None:
        if self.hidden_dim % self.n_heads:
            raise ValueError(f"hidden_dim {self.hidden_dim} is not divisible by n_heads {self.n_heads}")
        if self.n_heads % self.n_kv_heads:
            raise ValueError(f"n_heads {self.n_heads} is not divisible by n_kv_heads {self.n_kv_heads}")
        if self.head_dim % 2:
            raise ValueError(f"head_dim {self.head_dim} must be even for RoPE")


class KVCache:
    """Preallocated per-layer keys and values, ``(batch, kv_heads, max_len, head_dim)``."""

    def __init__(self, config: ModelConfig, batch: int, max_len: int, *, device, dtype) -> None:
        shape = (batch, config.n_kv_heads, max_len, config.head_dim)
        self.k = [torch.empty(shape, device=device, dtype=dtype) for _ in range(config.n_layers)]
        self.v = [torch.empty(shape, device=device, dtype=dtype) for _ in range(config.n_layers)]
        self.length = 0
        self.max_len = max_len

    def slot(self, layer: int, start: int, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Writable ``(batch, n, kv_heads, head_dim)`` views of positions ``[start, start + n)``."""
        if start + n > self.max_len:
            raise ValueError(f"KV cache holds {self.max_len} positions, asked for {start + n}")
        return (self.k[layer][:, :, start:start + n].transpose(1, 2),
                self.v[layer][:, :, start:start + n].transpose(1, 2))

    def view(self, layer: int, end: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.k[layer][:, :, :end], self.v[layer][:, :, :end]


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, backend: Backend) -> None:
        super().__init__()
        self.cfg = cfg
        self.backend = backend
        d, hd = cfg.hidden_dim, cfg.head_dim
        self.q_dim = cfg.n_heads * hd
        self.kv_dim = cfg.n_kv_heads * hd
        self.input_norm_weight = nn.Parameter(torch.ones(d))
        self.post_attention_norm_weight = nn.Parameter(torch.ones(d))
        self.qkv_proj = nn.Linear(d, self.q_dim + 2 * self.kv_dim, bias=False)
        self.o_proj = nn.Linear(self.q_dim, d, bias=False)
        self.gate_up_proj = nn.Linear(d, 2 * cfg.intermediate_dim, bias=False)
        self.down_proj = nn.Linear(cfg.intermediate_dim, d, bias=False)

    # -------------------------------------------------------- hot-path ops
    def _norm(self, x, residual, weight):
        eps = self.cfg.eps
        if self.backend == "b200":
            if residual is None:
                return kernels.rmsnorm_cuda_sm100(x, weight, eps), x
            return kernels.rmsnorm_residual_cuda_sm100(x, residual, weight, eps)
        if residual is None:
            return reference_ops().rmsnorm_ref(x, weight, eps), x
        return reference_ops().rmsnorm_residual_ref(x, residual, weight, eps)

    def _rope(self, q, k, cos, sin, k_dest):
        style = self.cfg.rope_style
        if self.backend == "b200":
            if k_dest is None:
                return kernels.rope_qk_cuda_sm100(q, k, cos, sin, style)
            q_out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
            rope_qk_into(q, k, cos, sin, style, q_out, k_dest)
            return q_out, k_dest
        q_out, k_out = reference_ops().rope_ref(q, cos, sin, style), reference_ops().rope_ref(k, cos, sin, style)
        if k_dest is not None:
            k_dest.copy_(k_out)
            k_out = k_dest
        return q_out, k_out

    def _swiglu(self, gu):
        f = self.cfg.intermediate_dim
        gate, up = gu[..., :f], gu[..., f:]
        if self.backend == "b200":
            return kernels.swiglu_cuda_sm100(gate, up)
        return reference_ops().swiglu_ref(gate, up)

    # --------------------------------------------------------------- block
    def forward(self, x, residual, cos, sin, cache: KVCache | None, layer: int):
        cfg = self.cfg
        b, s, _ = x.shape
        h, residual = self._norm(x, residual, self.input_norm_weight)
        qkv = self.qkv_proj(h)
        q = qkv[..., : self.q_dim].view(b, s, cfg.n_heads, cfg.head_dim)
        k = qkv[..., self.q_dim : self.q_dim + self.kv_dim].view(b, s, cfg.n_kv_heads, cfg.head_dim)
        v = qkv[..., self.q_dim + self.kv_dim :].view(b, s, cfg.n_kv_heads, cfg.head_dim)
        start = cache.length if cache is not None else 0
        if s > 1 and start > 0:
            raise NotImplementedError("chunked prefill onto a non-empty cache is not supported")
        k_dest = v_dest = None
        if cache is not None:
            k_dest, v_dest = cache.slot(layer, start, s)
        q, k = self._rope(q, k, cos, sin, k_dest)
        if cache is not None:
            v_dest.copy_(v)
            keys, values = cache.view(layer, start + s)
        else:
            keys, values = k.transpose(1, 2), v.transpose(1, 2)
        attn = F.scaled_dot_product_attention(
            q.transpose(1, 2), keys, values, is_causal=s > 1 and start == 0, enable_gqa=True
        )
        out = self.o_proj(attn.transpose(1, 2).reshape(b, s, self.q_dim))
        h, residual = self._norm(out, residual, self.post_attention_norm_weight)
        return self.down_proj(self._swiglu(self.gate_up_proj(h))), residual


    def forward_static(self, x, residual, cos, sin, cache: "KVCache", layer: int, pos: torch.Tensor,
                       mask: torch.Tensor):
        """One decode step with shapes fixed for CUDA-graph capture.

        ``pos`` is a one-element device tensor holding the write position; the
        new key and value go into the cache with ``index_copy_`` at ``pos`` and
        attention runs over the whole preallocated cache under ``mask``
        (``(1, 1, 1, max_len)``, true up to ``pos``), so nothing depends on
        host-side lengths.
        """
        cfg = self.cfg
        b = x.shape[0]
        h, residual = self._norm(x, residual, self.input_norm_weight)
        qkv = self.qkv_proj(h)
        q = qkv[..., : self.q_dim].view(b, 1, cfg.n_heads, cfg.head_dim)
        k = qkv[..., self.q_dim : self.q_dim + self.kv_dim].view(b, 1, cfg.n_kv_heads, cfg.head_dim)
        v = qkv[..., self.q_dim + self.kv_dim :].view(b, 1, cfg.n_kv_heads, cfg.head_dim)
        q, k = self._rope(q, k, cos, sin, None)
        cache.k[layer].index_copy_(2, pos, k.transpose(1, 2))
        cache.v[layer].index_copy_(2, pos, v.transpose(1, 2))
        attn = F.scaled_dot_product_attention(q.transpose(1, 2), cache.k[layer], cache.v[layer], attn_mask=mask,
                                              enable_gqa=True)
        out = self.o_proj(attn.transpose(1, 2).reshape(b, 1, self.q_dim))
        h, residual = self._norm(out, residual, self.post_attention_norm_weight)
        return self.down_proj(self._swiglu(self.gate_up_proj(h))), residual


class Decoder(nn.Module):
    """Embedding -> decoder stack -> final RMSNorm -> LM head."""

    def __init__(self, cfg: ModelConfig, backend: Backend = "b200") -> None:
        super().__init__()
        self.cfg = cfg
        self.backend = backend
        self.embed = nn.Embedding(cfg.vocab_size, cfg.hidden_dim)
        self.layers = nn.ModuleList(DecoderLayer(cfg, backend) for _ in range(cfg.n_layers))
        self.final_norm_weight = nn.Parameter(torch.ones(cfg.hidden_dim))
        self.lm_head = nn.Linear(cfg.hidden_dim, cfg.vocab_size, bias=False)
        self._tables: tuple[torch.Tensor, torch.Tensor] | None = None

    def rope_tables(self, device) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 tables for positions ``[0, max_seq_len)``, built once, sliced per call."""
        if self._tables is None or self._tables[0].device != torch.device(device):
            self._tables = reference_ops().build_rope_tables(self.cfg.max_seq_len, self.cfg.head_dim,
                                                  base=self.cfg.rope_base, device=device)
        return self._tables

    def new_cache(self, batch: int, max_len: int | None = None) -> KVCache:
        p = self.embed.weight
        return KVCache(self.cfg, batch, max_len or self.cfg.max_seq_len, device=p.device, dtype=p.dtype)

    def hidden(self, ids: torch.Tensor, cache: KVCache | None = None) -> torch.Tensor:
        """Final-normed hidden states ``(batch, seq, hidden)`` of token ids ``(batch, seq)``."""
        s = ids.shape[1]
        start = cache.length if cache is not None else 0
        cos, sin = self.rope_tables(ids.device)
        cos, sin = cos[start:start + s], sin[start:start + s]
        x = self.embed(ids)
        residual = None
        for i, layer in enumerate(self.layers):
            x, residual = layer(x, residual, cos, sin, cache, i)
        if cache is not None:
            cache.length = start + s
        if self.backend == "b200":
            out, _ = kernels.rmsnorm_residual_cuda_sm100(x, residual, self.final_norm_weight, self.cfg.eps)
        else:
            out, _ = reference_ops().rmsnorm_residual_ref(x, residual, self.final_norm_weight, self.cfg.eps)
        return out

    def forward(self, ids: torch.Tensor, cache: KVCache | None = None) -> torch.Tensor:
        """Logits of the last position of each sequence, ``(batch, vocab)``."""
        return self.lm_head(self.hidden(ids, cache)[:, -1])


class GraphDecoder:
    """Greedy decoding with each whole step captured in one CUDA graph.

    A step — embedding, every layer, final norm, LM head, argmax — is one graph
    replay: one launch instead of ~55, so the step runs at device speed rather
    than at the speed of Python issuing kernels. The position lives on the
    device and advances inside the graph; attention covers the preallocated
    cache under a position mask, so the graph is valid for every step. Tokens
    are written to ``tokens[:, step]`` on the device.
    """

    def __init__(self, model: "Decoder", cache: KVCache, first_token: torch.Tensor, steps: int) -> None:
        self.model = model
        self.cache = cache
        dev = first_token.device
        self.start = cache.length
        self.pos = torch.tensor([cache.length], dtype=torch.int64, device=dev)
        self.step_idx = torch.zeros(1, dtype=torch.int64, device=dev)
        self.tok = first_token.clone()
        self.tokens = torch.zeros(first_token.shape[0], steps, dtype=torch.int64, device=dev)
        self.arange = torch.arange(cache.max_len, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.steps = steps

    def _step(self) -> None:
        m = self.model
        cos_full, sin_full = m.rope_tables(self.tok.device)
        cos = cos_full.index_select(0, self.pos)
        sin = sin_full.index_select(0, self.pos)
        mask = (self.arange <= self.pos).view(1, 1, 1, -1)
        x = m.embed(self.tok)
        residual = None
        for i, layer in enumerate(m.layers):
            x, residual = layer.forward_static(x, residual, cos, sin, self.cache, i, self.pos, mask)
        if m.backend == "b200":
            h, _ = kernels.rmsnorm_residual_cuda_sm100(x, residual, m.final_norm_weight, m.cfg.eps)
        else:
            h, _ = reference_ops().rmsnorm_residual_ref(x, residual, m.final_norm_weight, m.cfg.eps)
        nxt = m.lm_head(h[:, -1]).argmax(-1, keepdim=True)
        self.tok.copy_(nxt)
        self.tokens.index_copy_(1, self.step_idx, nxt)
        self.pos.add_(1)
        self.step_idx.add_(1)

    def capture(self) -> None:
        """Warm up on a side stream, then capture one step (the state is reset after)."""
        self.reset()
        side = torch.cuda.Stream(self.tok.device)
        side.wait_stream(torch.cuda.current_stream(self.tok.device))
        with torch.cuda.stream(side):
            for _ in range(2):
                self._step()
        torch.cuda.current_stream(self.tok.device).wait_stream(side)
        self.reset()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        self.reset()

    def reset(self, first_token: torch.Tensor | None = None) -> None:
        self.pos.fill_(self.start)
        self.step_idx.zero_()
        if first_token is not None:
            self.tok.copy_(first_token)

    def run(self, first_token: torch.Tensor) -> torch.Tensor:
        """Greedy-decode ``steps`` tokens from the cached context; returns ``(batch, steps)``."""
        if self.graph is None:
            self.capture()
        self.reset(first_token)
        for _ in range(self.steps):
            self.graph.replay()
        return self.tokens


def build_decoder(cfg: ModelConfig, *, backend: Backend = "b200", device="cuda", dtype=torch.bfloat16,
                  seed: int = 0, std: float = 0.02) -> Decoder:
    """Decoder with reproducible N(0, std) projection/embedding weights and unit norm weights."""
    device = torch.device(device)
    with torch.device("meta"):
        model = Decoder(cfg, backend)
    model = model.to_empty(device=device).to(dtype)
    gen = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm_weight" in name:
                p.fill_(1.0)
            else:
                p.copy_(torch.randn(p.shape, generator=gen, device=device, dtype=torch.float32) * std)
    return model.eval()


def rope_qk_into(q, k, cos, sin, style, q_out, k_out) -> None:
    """``rope_qk`` writing into caller-provided views (e.g. a KV-cache slot).

    The same checks as ``rope_qk_cuda_sm100``, plus the outputs': every one of
    the four tensors is a CUDA tensor of q's dtype on q's device with a
    contiguous last axis (the kernel indexes all of them in q's element size),
    and each output has its input's shape.
    """
    fn = "rope_qk_into"
    if style not in kernels.ROPE_STYLES:
        raise ValueError(f"Unknown RoPE style '{style}', expected one of {kernels.ROPE_STYLES}")
    kernels._require_cuda(q, fn)
    kernels._check_rope_args(q, cos, sin, fn)
    kernels._check_rope_args(k, cos, sin, fn)
    code = kernels._dtype_code(q, "q", fn)
    for name, t in (("k", k), ("q_out", q_out), ("k_out", k_out)):
        if t.dtype != q.dtype or t.device != q.device:
            raise ValueError(f"{fn}: {name} must match q in dtype and device ({q.dtype} on {q.device})")
    for t in (q, k, q_out, k_out):
        if t.stride(-1) != 1:
            raise ValueError(f"{fn}: tensors with a contiguous last axis required")
    if q_out.shape != q.shape or k_out.shape != k.shape:
        raise ValueError(f"{fn}: output shapes must match the inputs")
    if k.shape[:2] != q.shape[:2] or k.shape[-1] != q.shape[-1]:
        raise ValueError(f"{fn}: q {tuple(q.shape)} and k {tuple(k.shape)} must share batch, seq_len, head_dim")
    cos, sin = kernels._rope_tables(cos, sin)
    b, s, qh, d = q.shape
    with kernels._DeviceGuard(q.device):
        status = _native.active().ako_b200_rope_qk(
            q.data_ptr(), q.stride(0), q.stride(1), q.stride(2),
            k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
            cos.data_ptr(), sin.data_ptr(), cos.stride(0),
            q_out.data_ptr(), q_out.stride(0), q_out.stride(1), q_out.stride(2),
            k_out.data_ptr(), k_out.stride(0), k_out.stride(1), k_out.stride(2),
            b, s, qh, k.shape[2], d, kernels._STYLE_CODE[style], code, kernels._stream(q.device),
        )
    _native.raise_for_status(status, fn)
