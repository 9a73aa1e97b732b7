"""PyTorch statement of the operators' math, exported for API compatibility.

The reference project ships these three functions as ``*_reference``
(``sm120_rmsnorm/reference.py`` there) and code written against it imports
them from the package, so they keep their names here. They define the
rounding order the CUDA kernels follow and run on whatever device their
inputs live on. The operators in ``ops.py`` never call them.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm_reference(
    x: torch.Tensor,
    weight: torch.Tensor,
    epsilon: float = 1e-6,
) -> torch.Tensor:
    """``x * rsqrt(mean(x^2) + eps) * weight`` in fp32, cast back to ``x.dtype``."""
    wide = x.float()
    inv_rms = torch.rsqrt(wide.square().mean(dim=-1, keepdim=True) + epsilon)
    return (wide * inv_rms * weight.float()).to(x.dtype)


def fused_add_rms_norm_reference(
    x: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    epsilon: float = 1e-6,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Return ``(RMSNorm(x + residual) * weight, x + residual)``; the sum is
    rounded to the activation dtype before it is normalised."""
    summed = x + residual
    return rms_norm_reference(summed, weight, epsilon), summed


def qk_rms_norm_rope_reference(
    query: torch.Tensor,
    key: torch.Tensor,
    query_weight: torch.Tensor,
    key_weight: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    epsilon: float = 1e-6,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-head RMSNorm (rounded to the activation dtype, times the weight in
    that dtype) followed by half-split RoPE in fp32, for ``[tokens, heads, D]``
    query and key. ``cos_sin_cache`` is ``[P, D]`` or ``[P, 1, D]`` with cos in
    the first half of the last dimension and sin in the second."""
    width = cos_sin_cache.shape[-1]
    rows = cos_sin_cache.reshape(-1, width)[positions].unsqueeze(-2)  # [T, 1, D]
    cos, sin = rows.chunk(2, dim=-1)

    def rotate(t: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        normed = F.rms_norm(t.float(), (t.shape[-1],), None, epsilon).to(t.dtype) * weight
        first, second = normed.float().chunk(2, dim=-1)
        return torch.cat((first * cos - second * sin, second * cos + first * sin),
                         dim=-1).to(t.dtype)

    return rotate(query, query_weight), rotate(key, key_weight)
