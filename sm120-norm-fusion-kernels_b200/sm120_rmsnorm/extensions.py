"""Engine-side extensions of the same hot path, beyond the reference's API.

The reference's operators (``sm120_rmsnorm.ops``) stay exactly as they are.
These cover what an inference engine around them needs, on the same B200
kernels' numerics (csrc/head_cache.cu, csrc/norm_quant.cu):

* :func:`qk_norm_rope_cache_` -- per-head Q/K RMSNorm + RoPE + paged KV store
  for head sizes 64 / 128 / 256, partial rotary, NEOX or interleaved pairs,
  Q/K/V as strided views of one QKV projection output, NHD or HND caches of
  any block size, and fp8 e4m3 caches with per-tensor scales. With
  head_dim = rotary_dim = 128, NEOX, a same-dtype NHD cache and dense inputs it
  is bit-identical to ``ops.fused_qk_rms_norm_rope_kv``.
* :func:`rms_norm_static_fp8_quant`, :func:`fused_add_rms_norm_static_fp8_quant`,
  :func:`rms_norm_dynamic_per_token_quant` -- RMSNorm (after the optional
  residual add) with an fp8 e4m3 output: the row y is computed with the
  rounding sequence of ``ops.rms_norm`` / ``ops.fused_add_rms_norm`` and then
  quantised:
  static ``q = sat(y * (1 / scale))``; dynamic per row
  ``scale = max(min(max|y|, scale_ub) / 448, 1 / (448 * 512))`` and
  ``q = sat(y * (1 / scale))``, sat() clamping to +-448 and rounding to nearest
  even. The operator names and argument order are the ones fp8 inference
  engines use for these fusions.
* :func:`rms_norm_nvfp4_quant` -- the same RMSNorm quantised to NVFP4 (e2m1
  values, one e4m3 scale per 16 elements, a caller-supplied global scale),
  with the block scales row-major or in the tiled layout of block-scaled
  tensor-core GEMMs.

Registered as ``torch.ops.sm120_norm_ext.*``; no fallback when the extension
is missing.
"""
from __future__ import annotations

import torch

from .ops import _C, _extension

FP8_MAX = 448.0
MIN_TOKEN_SCALE = 1.0 / (448.0 * 512.0)


def qk_norm_rope_cache_(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor | None,
    query_weight: torch.Tensor,
    key_weight: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    key_cache: torch.Tensor | None = None,
    value_cache: torch.Tensor | None = None,
    slot_mapping: torch.Tensor | None = None,
    k_scale: torch.Tensor | None = None,
    v_scale: torch.Tensor | None = None,
    is_neox: bool = True,
    kv_cache_layout: str = "NHD",
    epsilon: float = 1e-6,
) -> None:
    """In place on ``query`` [T, Hq, D] and ``key`` [T, Hk, D] (any token
    stride, heads adjacent): per-head RMSNorm with the reference's double
    rounding, then RoPE on the first ``cos_sin_cache.size(-1)`` elements.
    With caches ([blocks, block_size, Hk, D] for "NHD", [blocks, Hk,
    block_size, D] for "HND"; activation dtype, or float8_e4m3fn / uint8 with
    one-element float32 ``k_scale`` / ``v_scale``), the rotated K and ``value``
    are stored at ``slot_mapping`` (int32; slots outside the cache skipped)."""
    _extension()
    torch.ops.sm120_norm_ext.qk_norm_rope_cache_(
        query, key, value, query_weight, key_weight, positions, cos_sin_cache, key_cache,
        value_cache, slot_mapping, k_scale, v_scale, is_neox, kv_cache_layout, epsilon)


def rms_norm_static_fp8_quant(result: torch.Tensor, input: torch.Tensor, weight: torch.Tensor,
                              scale: torch.Tensor, epsilon: float = 1e-6) -> None:
    """``result`` (float8_e4m3fn, shape of ``input``) = sat(rms_norm(input) * (1 / scale))."""
    _extension()
    torch.ops.sm120_norm_ext.rms_norm_static_fp8_quant(result, input, weight, scale, epsilon)


def fused_add_rms_norm_static_fp8_quant(result: torch.Tensor, input: torch.Tensor,
                                        residual: torch.Tensor, weight: torch.Tensor,
                                        scale: torch.Tensor, epsilon: float = 1e-6) -> None:
    """``residual`` = input + residual (in place); ``result`` =
    sat(rms_norm(residual) * (1 / scale)). ``input`` is not modified."""
    _extension()
    torch.ops.sm120_norm_ext.fused_add_rms_norm_static_fp8_quant(
        result, input, residual, weight, scale, epsilon)


def rms_norm_dynamic_per_token_quant(result: torch.Tensor, input: torch.Tensor,
                                     weight: torch.Tensor, scale: torch.Tensor,
                                     epsilon: float = 1e-6, scale_ub: torch.Tensor | None = None,
                                     residual: torch.Tensor | None = None) -> None:
    """Per-row dynamic scales into ``scale`` (float32, one per row) and the
    quantised rows into ``result``; with ``residual``, the residual add happens
    first and ``residual`` is updated in place."""
    _extension()
    torch.ops.sm120_norm_ext.rms_norm_dynamic_per_token_quant(
        result, input, weight, scale, epsilon, scale_ub, residual)


def rms_norm_nvfp4_quant(result: torch.Tensor, block_scale: torch.Tensor, input: torch.Tensor,
                         weight: torch.Tensor, global_scale: torch.Tensor, epsilon: float = 1e-6,
                         residual: torch.Tensor | None = None,
                         swizzled_scales: bool = True) -> None:
    """RMSNorm (after the residual add when ``residual`` is given, which is
    then updated in place) quantised to NVFP4 for a block-scaled fp4 GEMM.
    Per 16 elements of a row, with g = ``global_scale``:
    ``s = e4m3(g * (max|y| * fp32(1/6)))``, ``q = e2m1(y * (g / s))`` (nearest even,
    saturating). ``result``: ``[rows, hidden / 2]`` uint8, element 2i in the
    low nibble; ``block_scale``: the e4m3 scales, row-major
    ``[rows, hidden / 16]`` or, when ``swizzled_scales``, the 128 x 4 tiled
    layout tensor-core GEMMs read (``round_up(rows, 128) *
    round_up(hidden / 16, 4)`` bytes, padding untouched)."""
    _extension()
    torch.ops.sm120_norm_ext.rms_norm_nvfp4_quant(result, block_scale, input, weight,
                                                  global_scale, epsilon, residual,
                                                  swizzled_scales)


def qkv_proj_norm_rope_cache_(hidden: torch.Tensor, qkv_weight: torch.Tensor,
                              qkv: torch.Tensor, query_heads: int, key_heads: int,
                              query_weight: torch.Tensor | None = None,
                              key_weight: torch.Tensor | None = None,
                              positions: torch.Tensor | None = None,
                              cos_sin_cache: torch.Tensor | None = None,
                              key_cache: torch.Tensor | None = None,
                              value_cache: torch.Tensor | None = None,
                              slot_mapping: torch.Tensor | None = None,
                              epsilon: float = 1e-6, fuse_norm: bool = True) -> None:
    """``qkv = hidden @ qkv_weight.T`` on the tensor cores (bf16, fp32
    accumulation) into ``qkv`` ``[tokens, (Hq + 2Hk) * 128]``; with
    ``fuse_norm`` the epilogue then applies, per head, exactly what
    ``ops.fused_qk_rms_norm_rope_kv`` does to the ``[tokens, heads, 128]`` view
    of ``qkv`` (Q/K norm + RoPE in place, rotated K and V into the caches at
    ``slot_mapping`` when caches are given)."""
    _extension()
    torch.ops.sm120_norm_ext.qkv_proj_norm_rope_cache_(
        hidden, qkv_weight, qkv, query_heads, key_heads, query_weight, key_weight, positions,
        cos_sin_cache, key_cache, value_cache, slot_mapping, epsilon, fuse_norm)


def nvfp4_scale_bytes(rows: int, hidden: int, swizzled_scales: bool = True) -> int:
    """Bytes of the block-scale buffer for ``rows`` x ``hidden``."""
    blocks = hidden // 16
    if not swizzled_scales:
        return rows * blocks
    return (rows + 127) // 128 * 128 * ((blocks + 3) // 4 * 4)


if _C is not None:
    # Meta implementations: every operator only mutates its arguments.

    @torch.library.register_fake("sm120_norm_ext::qk_norm_rope_cache_")
    def _qk_norm_rope_cache_meta(query, key, value, query_weight, key_weight, positions,
                                 cos_sin_cache, key_cache, value_cache, slot_mapping, k_scale,
                                 v_scale, is_neox=True, kv_cache_layout="NHD",
                                 epsilon=1e-6) -> None:
        return None

    @torch.library.register_fake("sm120_norm_ext::rms_norm_static_fp8_quant")
    def _rms_norm_static_fp8_quant_meta(result, input, weight, scale, epsilon) -> None:
        return None

    @torch.library.register_fake("sm120_norm_ext::fused_add_rms_norm_static_fp8_quant")
    def _fused_add_rms_norm_static_fp8_quant_meta(result, input, residual, weight, scale,
                                                  epsilon) -> None:
        return None

    @torch.library.register_fake("sm120_norm_ext::rms_norm_dynamic_per_token_quant")
    def _rms_norm_dynamic_per_token_quant_meta(result, input, weight, scale, epsilon,
                                               scale_ub=None, residual=None) -> None:
        return None

    @torch.library.register_fake("sm120_norm_ext::rms_norm_nvfp4_quant")
    def _rms_norm_nvfp4_quant_meta(result, block_scale, input, weight, global_scale,
                                   epsilon=1e-6, residual=None, swizzled_scales=True) -> None:
        return None

    @torch.library.register_fake("sm120_norm_ext::qkv_proj_norm_rope_cache_")
    def _qkv_proj_norm_rope_cache_meta(hidden, qkv_weight, qkv, query_heads, key_heads,
                                       query_weight=None, key_weight=None, positions=None,
                                       cos_sin_cache=None, key_cache=None, value_cache=None,
                                       slot_mapping=None, epsilon=1e-6, fuse_norm=True) -> None:
        return None
