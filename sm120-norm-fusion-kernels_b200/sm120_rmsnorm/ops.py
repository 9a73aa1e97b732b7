"""Public operators: the reference's ``sm120_rmsnorm.ops`` API on B200 kernels.

Same names, argument order, defaults and error behaviour as the reference
project's ``sm120_rmsnorm/ops.py``; each call goes to the compiled ``_C``
extension (csrc/torch_binding.cpp), which validates the tensors and calls the
C ABI (include/sm120norm_b200.h). There is no fallback: if the extension is
not built every operator raises ``RuntimeError``.

``version`` keeps the reference's accepted values; on B200 they select launch
shapes of the sm_100a kernels and all give the same results:

========================  ==========  =========================================
operator                  default     accepted values
========================  ==========  =========================================
rms_norm(_out)            2           1 (block per row), 2 (B200 shape dispatch)
fused_add_rms_norm*       0           0 (B200 shape dispatch), 2 (block per row,
                                      any hidden size), 3 (warp per row) and
                                      4 (one 16-byte pack per thread); 3 and 4
                                      need hidden_size=1024
fused_qk_rms_norm_rope    2           1 (two warps per block), 2 (B200 default)
fused_qk_rms_norm_rope_kv 1           1 (B200 default), 4 (four warps per block)
========================  ==========  =========================================
"""
from __future__ import annotations

import torch

try:
    from . import _C
except ImportError as _error:  # the shared libraries are not built
    _C = None
    _IMPORT_ERROR: ImportError | None = _error
else:
    _IMPORT_ERROR = None


def _extension():
    if _C is None:
        raise RuntimeError(
            "the sm120_rmsnorm CUDA extension is not built; run "
            "`python sm120-norm-fusion-kernels_b200/build.py` (or __graft_entry__.build())"
        ) from _IMPORT_ERROR
    return _C


def rms_norm(
    x: torch.Tensor,
    weight: torch.Tensor,
    epsilon: float = 1e-6,
    version: int = 2,
) -> torch.Tensor:
    """RMSNorm over the last dimension into a new tensor."""
    return _extension().rms_norm(x, weight, epsilon, version)


def rms_norm_out(
    x: torch.Tensor,
    weight: torch.Tensor,
    output: torch.Tensor,
    epsilon: float = 1e-6,
    version: int = 2,
) -> None:
    """RMSNorm over the last dimension into ``output``."""
    _extension().rms_norm_out(x, weight, output, epsilon, version)


def fused_add_rms_norm(
    x: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    epsilon: float = 1e-6,
    version: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Return ``(RMSNorm(x + residual) * weight, x + residual)``."""
    output, residual_output = _extension().fused_add_rms_norm(x, residual, weight, epsilon, version)
    return output, residual_output


def fused_add_rms_norm_out(
    x: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    output: torch.Tensor,
    residual_output: torch.Tensor,
    epsilon: float = 1e-6,
    version: int = 0,
) -> None:
    """Write ``x + residual`` to ``residual_output`` and its RMSNorm to ``output``."""
    _extension().fused_add_rms_norm_out(
        x, residual, weight, output, residual_output, epsilon, version)


def fused_add_rms_norm_inplace(
    x: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    epsilon: float = 1e-6,
    version: int = 0,
) -> None:
    """``residual += x``; ``x = RMSNorm(residual) * weight`` (vLLM / FlashInfer contract)."""
    _extension().fused_add_rms_norm_inplace(x, residual, weight, epsilon, version)


def fused_qk_rms_norm_rope(
    query: torch.Tensor,
    key: torch.Tensor,
    query_weight: torch.Tensor,
    key_weight: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    epsilon: float = 1e-6,
    version: int = 2,
) -> None:
    """Per-head RMSNorm then half-split RoPE on ``query`` and ``key``, in place.

    Dispatched through ``torch.ops.sm120_norm`` so torch.compile and CUDA
    graphs see one opaque mutating operator.
    """
    _extension()
    torch.ops.sm120_norm.fused_qk_rms_norm_rope_(
        query, key, query_weight, key_weight, positions, cos_sin_cache, epsilon, version)


def fused_qk_rms_norm_rope_kv(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    query_weight: torch.Tensor,
    key_weight: torch.Tensor,
    positions: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    epsilon: float = 1e-6,
    version: int = 1,
) -> None:
    """As :func:`fused_qk_rms_norm_rope`, then store rotated K and V into the
    paged cache at ``slot_mapping`` (negative slots are padding and skipped)."""
    _extension()
    torch.ops.sm120_norm.fused_qk_rms_norm_rope_kv_(
        query, key, value, query_weight, key_weight, positions, cos_sin_cache,
        key_cache, value_cache, slot_mapping, epsilon, version)


if _C is not None:
    # Meta implementations: both operators only mutate their inputs.

    @torch.library.register_fake("sm120_norm::fused_qk_rms_norm_rope_")
    def _qk_rms_norm_rope_meta(query, key, query_weight, key_weight, positions,
                               cos_sin_cache, epsilon=1e-6, version=2) -> None:
        return None

    @torch.library.register_fake("sm120_norm::fused_qk_rms_norm_rope_kv_")
    def _qk_rms_norm_rope_kv_meta(query, key, value, query_weight, key_weight, positions,
                                  cos_sin_cache, key_cache, value_cache, slot_mapping,
                                  epsilon=1e-6, version=1) -> None:
        return None
