"""Engine-side caller of the hot path: the attention prologue of a Qwen3
decoder layer, as an inference engine runs it around these operators.

Per layer (reference project, README.md:11-12, where the same two operators
are called from a decode engine's Qwen3 layer):

1. ``fused_add_rms_norm_inplace(hidden, residual, input_norm_weight)`` --
   residual += hidden; hidden = RMSNorm(residual) (in place);
2. ``qkv = hidden @ qkv_weight.T`` -- the QKV projection, a plain library
   GEMM (cuBLAS through PyTorch) into a preallocated buffer;
3. ``qk_norm_rope_cache_`` on strided Q / K / V views of ``qkv`` -- per-head
   Q/K RMSNorm + RoPE in place and the paged KV store, with no gather copies
   (the reference's kernel needs contiguous Q / K, so an engine built on it
   copies them out first).

With ``fused_projection=True`` steps 2 and 3 are one kernel: the QKV
projection on the tensor cores with the Q/K norm + RoPE + KV store in its
epilogue (``extensions.qkv_proj_norm_rope_cache_``; bf16, head_dim 128, dense
NHD caches), bit-identical to that kernel's plain GEMM followed by step 3.

:class:`DecodeGraph` captures the prologues of all layers of one decode step
into a single CUDA graph, so the host launches one graph per step; the B200
kernels additionally overlap each launch with the tail of the previous kernel
(programmatic dependent launch).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import extensions, ops


@dataclass(frozen=True)
class Qwen3AttentionShape:
    hidden: int = 4096
    query_heads: int = 32
    key_heads: int = 8
    head_dim: int = 128
    rope_theta: float = 1e6
    max_positions: int = 32768
    epsilon: float = 1e-6

    @property
    def qkv_width(self) -> int:
        return (self.query_heads + 2 * self.key_heads) * self.head_dim


def rope_cos_sin_cache(shape: Qwen3AttentionShape, device, rotary_dim: int | None = None):
    """fp32 [max_positions, rotary_dim]: cos | sin of position * theta^(-2i/d)."""
    rotary_dim = rotary_dim or shape.head_dim
    inv = 1.0 / (shape.rope_theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32,
                                                    device=device) / rotary_dim))
    f = torch.outer(torch.arange(shape.max_positions, dtype=torch.float32, device=device), inv)
    return torch.cat((f.cos(), f.sin()), dim=-1)


class Qwen3AttentionPrologue:
    """Weights and the per-layer call. ``forward`` returns the (strided) Q, K
    and V views into the layer's QKV buffer; K and V are also in the cache."""

    def __init__(self, shape: Qwen3AttentionShape, device, dtype=torch.bfloat16,
                 generator: torch.Generator | None = None):
        self.shape = shape
        g = generator
        std = 1.0 / math.sqrt(shape.hidden)
        self.input_norm_weight = (1 + 0.1 * torch.randn(shape.hidden, device=device,
                                                        generator=g)).to(dtype)
        self.qkv_weight = (std * torch.randn(shape.qkv_width, shape.hidden, device=device,
                                             generator=g)).to(dtype)
        self.query_norm_weight = (1 + 0.1 * torch.randn(shape.head_dim, device=device,
                                                        generator=g)).to(dtype)
        self.key_norm_weight = (1 + 0.1 * torch.randn(shape.head_dim, device=device,
                                                      generator=g)).to(dtype)

    def split(self, qkv: torch.Tensor):
        s = self.shape
        t = qkv.shape[0]
        q_end = s.query_heads * s.head_dim
        k_end = q_end + s.key_heads * s.head_dim
        return (qkv[:, :q_end].view(t, s.query_heads, s.head_dim),
                qkv[:, q_end:k_end].view(t, s.key_heads, s.head_dim),
                qkv[:, k_end:].view(t, s.key_heads, s.head_dim))

    def forward(self, hidden: torch.Tensor, residual: torch.Tensor, positions: torch.Tensor,
                cos_sin_cache: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                slot_mapping: torch.Tensor, qkv_out: torch.Tensor, k_scale=None, v_scale=None,
                kv_cache_layout: str = "NHD", fused_projection: bool = False):
        s = self.shape
        ops.fused_add_rms_norm_inplace(hidden, residual, self.input_norm_weight, s.epsilon)
        if fused_projection:
            extensions.qkv_proj_norm_rope_cache_(
                hidden, self.qkv_weight, qkv_out, s.query_heads, s.key_heads,
                self.query_norm_weight, self.key_norm_weight, positions, cos_sin_cache,
                key_cache, value_cache, slot_mapping, s.epsilon)
            return self.split(qkv_out)
        torch.matmul(hidden, self.qkv_weight.t(), out=qkv_out)
        q, k, v = self.split(qkv_out)
        extensions.qk_norm_rope_cache_(
            q, k, v, self.query_norm_weight, self.key_norm_weight, positions, cos_sin_cache,
            key_cache, value_cache, slot_mapping, k_scale, v_scale, True, kv_cache_layout,
            s.epsilon)
        return q, k, v


class DecodeGraph:
    """The prologues of ``layers`` decoder layers for one decode batch,
    captured once as a CUDA graph over static buffers. Between layers the
    hidden state for the next layer is the previous QKV buffer's first
    ``hidden`` columns (a stand-in for attention + output projection + MLP,
    which are not part of this path), so every layer reads fresh data.

    Fill ``hidden``, ``residual``, ``positions`` and ``slot_mapping`` in
    place, then ``replay()``. ``fused_projection`` None picks the fused
    projection where it measured faster (:meth:`fused_projection_pays`).
    """

    def __init__(self, layers: list[Qwen3AttentionPrologue], batch: int, cos_sin_cache,
                 key_caches: list[torch.Tensor], value_caches: list[torch.Tensor],
                 k_scale=None, v_scale=None, kv_cache_layout: str = "NHD",
                 fused_projection: bool | None = None):
        shape = layers[0].shape
        if shape.qkv_width < shape.hidden:
            raise ValueError("the stand-in between layers needs qkv_width >= hidden")
        dev = cos_sin_cache.device
        dtype = layers[0].qkv_weight.dtype
        if fused_projection is None:
            fused_projection = self.fused_projection_pays(batch, shape, dtype, key_caches,
                                                          k_scale, kv_cache_layout)
        self.fused_projection = fused_projection
        self.layers = layers
        self.hidden = torch.zeros(batch, shape.hidden, device=dev, dtype=dtype)
        self.residual = torch.zeros_like(self.hidden)
        self.positions = torch.zeros(batch, device=dev, dtype=torch.int64)
        self.slot_mapping = torch.full((batch,), -1, device=dev, dtype=torch.int32)
        self.qkv = [torch.empty(batch, shape.qkv_width, device=dev, dtype=dtype) for _ in layers]
        self.layer_hidden = [torch.empty_like(self.hidden) for _ in layers[1:]]
        self._args = (cos_sin_cache, key_caches, value_caches, k_scale, v_scale, kv_cache_layout,
                      fused_projection)
        self._run()  # load kernels and pick cuBLAS algorithms before capture
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._run()

    @staticmethod
    def fused_projection_pays(batch, shape, dtype, key_caches, k_scale, kv_cache_layout) -> bool:
        """Whether the projection with the fused Q/K epilogue is the faster
        choice: up to four tokens, where it streams the weights on the CUDA
        cores (a Qwen3-8B-shaped batch-1 step: 139.9 us against 166.8 us for
        cuBLAS followed by the Q/K kernel), and only where it applies (bf16,
        head_dim 128, dense bf16 NHD caches). From 16 tokens up cuBLAS followed
        by the Q/K kernel measured faster."""
        return (batch <= 4 and dtype == torch.bfloat16 and shape.head_dim == 128
                and kv_cache_layout == "NHD" and k_scale is None
                and all(c.dtype == torch.bfloat16 and c.is_contiguous() for c in key_caches))

    def _run(self):
        cos_sin, key_caches, value_caches, k_scale, v_scale, layout, fused = self._args
        hidden = self.hidden
        for i, layer in enumerate(self.layers):
            layer.forward(hidden, self.residual, self.positions, cos_sin, key_caches[i],
                          value_caches[i], self.slot_mapping, self.qkv[i], k_scale, v_scale,
                          layout, fused)
            if i + 1 < len(self.layers):
                nxt = self.layer_hidden[i]
                nxt.copy_(self.qkv[i][:, :layer.shape.hidden])
                hidden = nxt

    def replay(self):
        self.graph.replay()
