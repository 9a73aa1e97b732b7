"""B200 (sm_100a) fused normalisation kernels behind the ``sm120_rmsnorm`` API.

Drop-in for the reference package of the same name: the seven operators and
the three ``*_reference`` functions keep their names and signatures. The
kernels live in a C-ABI shared library (``libsm120norm_b200.so``, see
``include/sm120norm_b200.h``); ``_C`` binds it for PyTorch and ``capi`` binds
it with ctypes.
"""
from .ops import (
    fused_add_rms_norm,
    fused_add_rms_norm_inplace,
    fused_add_rms_norm_out,
    fused_qk_rms_norm_rope,
    fused_qk_rms_norm_rope_kv,
    rms_norm,
    rms_norm_out,
)
from .reference import (
    fused_add_rms_norm_reference,
    qk_rms_norm_rope_reference,
    rms_norm_reference,
)

__all__ = [
    "fused_add_rms_norm",
    "fused_add_rms_norm_reference",
    "fused_add_rms_norm_inplace",
    "fused_add_rms_norm_out",
    "fused_qk_rms_norm_rope",
    "fused_qk_rms_norm_rope_kv",
    "qk_rms_norm_rope_reference",
    "rms_norm",
    "rms_norm_out",
    "rms_norm_reference",
]
