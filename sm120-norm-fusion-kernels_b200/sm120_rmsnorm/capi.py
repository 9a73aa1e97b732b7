"""ctypes binding of the C ABI in ``include/sm120norm_b200.h``.

For callers that hold raw device pointers (another runtime, another language's
FFI, a custom allocator) rather than PyTorch tensors. Every function takes
integer device addresses, sizes and a ``cudaStream_t`` as an integer (0 = the
legacy default stream) and raises :class:`CApiError` on a non-zero status.
The library is loaded from this package directory.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY_NAME = "libsm120norm_b200.so"
LIBRARY_PATH = Path(__file__).resolve().parent / LIBRARY_NAME

F32, F16, BF16 = 0, 1, 2
OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3
ROPE_NEOX, ROPE_INTERLEAVED = 0, 1
CACHE_AUTO, CACHE_FP8_E4M3 = 0, 1
SCALES_ROW_MAJOR, SCALES_TILED_128X4 = 0, 1


class QkCacheArgs(ctypes.Structure):
    """``sm120n_qk_cache_args`` (include/sm120norm_b200.h), field for field."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("dtype", ctypes.c_int32),
        ("tokens", ctypes.c_int64),
        ("query_heads", ctypes.c_int64),
        ("key_heads", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("rotary_dim", ctypes.c_int64),
        ("rope_style", ctypes.c_int32),
        ("cache_dtype", ctypes.c_int32),
        ("query", ctypes.c_void_p),
        ("query_token_stride", ctypes.c_int64),
        ("key", ctypes.c_void_p),
        ("key_token_stride", ctypes.c_int64),
        ("value", ctypes.c_void_p),
        ("value_token_stride", ctypes.c_int64),
        ("query_weight", ctypes.c_void_p),
        ("key_weight", ctypes.c_void_p),
        ("positions", ctypes.c_void_p),
        ("cos_sin_cache", ctypes.c_void_p),
        ("rope_positions", ctypes.c_int64),
        ("key_cache", ctypes.c_void_p),
        ("value_cache", ctypes.c_void_p),
        ("slot_mapping", ctypes.c_void_p),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int64),
        ("cache_block_stride", ctypes.c_int64),
        ("cache_slot_stride", ctypes.c_int64),
        ("cache_head_stride", ctypes.c_int64),
        ("k_scale", ctypes.c_void_p),
        ("v_scale", ctypes.c_void_p),
        ("epsilon", ctypes.c_float),
    ]

    def __init__(self, **fields):
        fields.setdefault("epsilon", 1e-6)
        super().__init__(struct_size=ctypes.sizeof(QkCacheArgs), **fields)


# Every symbol include/sm120norm_b200.h declares, with its ctypes signature.
_i64, _i32, _f32, _vp = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p
SIGNATURES: dict[str, tuple[list, object]] = {
    "sm120n_abi_version": ([], _i32),
    "sm120n_last_error": ([], ctypes.c_char_p),
    "sm120n_status_string": ([_i32], ctypes.c_char_p),
    "sm120n_set_programmatic_launch": ([_i32], None),
    "sm120n_get_programmatic_launch": ([], _i32),
    "sm120n_get_device_faults": ([ctypes.POINTER(ctypes.c_uint32)], _i32),
    "sm120n_reset_device_faults": ([], _i32),
    "sm120n_set_wait_limit": ([ctypes.c_uint32], None),
    "sm120n_get_wait_limit": ([], ctypes.c_uint32),
    "sm120n_rms_norm": ([_vp, _vp, _vp, _i64, _i64, _i32, _f32, _i32, _vp], _i32),
    "sm120n_fused_add_rms_norm": ([_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _f32, _i32, _vp], _i32),
    "sm120n_fused_qk_rms_norm_rope": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _f32, _i32, _vp], _i32),
    "sm120n_fused_qk_rms_norm_rope_kv": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
         _i64, _i64, _i64, _i64, _i64, _i64, _i32, _f32, _i32, _vp], _i32),
    "sm120n_qk_norm_rope_cache": ([ctypes.POINTER(QkCacheArgs), _vp], _i32),
    "sm120n_rms_norm_fp8_quant": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _f32, _vp], _i32),
    "sm120n_rms_norm_fp4_quant": (
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _f32, _i32, _vp], _i32),
    "sm120n_qkv_proj_norm_rope_cache": (
        [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _i64,
         _f32, _i32, _vp], _i32),
}


class CApiError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message or f"status {status}")
        self.status = status


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load(path: str | Path | None = None) -> ctypes.CDLL:
    """Load (once) and return the shared library with typed signatures."""
    global _lib
    with _lock:
        if _lib is None or path is not None:
            lib = ctypes.CDLL(str(path or LIBRARY_PATH))
            for name, (argtypes, restype) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = lib
    return _lib


def _check(status: int) -> None:
    if status != OK:
        raise CApiError(status, load().sm120n_last_error().decode())


def abi_version() -> int:
    return load().sm120n_abi_version()


def set_programmatic_launch(enabled: bool) -> None:
    load().sm120n_set_programmatic_launch(1 if enabled else 0)


def device_faults() -> int:
    count = ctypes.c_uint32(0)
    _check(load().sm120n_get_device_faults(ctypes.byref(count)))
    return int(count.value)


def reset_device_faults() -> None:
    _check(load().sm120n_reset_device_faults())


class DeviceFaultError(RuntimeError):
    """A kernel gave up waiting on its own asynchronous copies and left rows
    unwritten (see :func:`check_device_faults`)."""


def check_device_faults(reset: bool = True) -> None:
    """Raise :class:`DeviceFaultError` when a bounded wait expired on the
    current device since the last reset (synchronises the device; the
    operators themselves stay asynchronous and never read the counter). With
    ``reset`` the counter is cleared before raising."""
    count = device_faults()
    if count:
        if reset:
            reset_device_faults()
        raise DeviceFaultError(f"{count} bounded wait(s) on asynchronous copies expired; the "
                               "affected rows of those calls were not written")


def set_wait_limit(polls: int) -> None:
    """Diagnostic: polls a kernel makes while waiting for its own bulk copies
    before it records an expired wait (0 restores the default)."""
    load().sm120n_set_wait_limit(int(polls))


def wait_limit() -> int:
    return int(load().sm120n_get_wait_limit())


def rms_norm(input_ptr, weight_ptr, output_ptr, rows, hidden_size, dtype, epsilon=1e-6,
             version=2, stream=0) -> None:
    _check(load().sm120n_rms_norm(input_ptr, weight_ptr, output_ptr, rows, hidden_size, dtype,
                                  epsilon, version, stream))


def fused_add_rms_norm(input_ptr, residual_ptr, weight_ptr, output_ptr, residual_output_ptr,
                       rows, hidden_size, dtype, epsilon=1e-6, version=0, stream=0) -> None:
    _check(load().sm120n_fused_add_rms_norm(input_ptr, residual_ptr, weight_ptr, output_ptr,
                                            residual_output_ptr, rows, hidden_size, dtype,
                                            epsilon, version, stream))


def fused_qk_rms_norm_rope(query_ptr, key_ptr, query_weight_ptr, key_weight_ptr, positions_ptr,
                           cos_sin_ptr, tokens, query_heads, key_heads, head_dim,
                           rope_positions, dtype, epsilon=1e-6, version=2, stream=0) -> None:
    _check(load().sm120n_fused_qk_rms_norm_rope(
        query_ptr, key_ptr, query_weight_ptr, key_weight_ptr, positions_ptr, cos_sin_ptr, tokens,
        query_heads, key_heads, head_dim, rope_positions, dtype, epsilon, version, stream))


def fused_qk_rms_norm_rope_kv(query_ptr, key_ptr, value_ptr, query_weight_ptr, key_weight_ptr,
                              positions_ptr, cos_sin_ptr, key_cache_ptr, value_cache_ptr,
                              slot_mapping_ptr, tokens, query_heads, key_heads, head_dim,
                              rope_positions, cache_slots, dtype, epsilon=1e-6, version=1,
                              stream=0) -> None:
    _check(load().sm120n_fused_qk_rms_norm_rope_kv(
        query_ptr, key_ptr, value_ptr, query_weight_ptr, key_weight_ptr, positions_ptr,
        cos_sin_ptr, key_cache_ptr, value_cache_ptr, slot_mapping_ptr, tokens, query_heads,
        key_heads, head_dim, rope_positions, cache_slots, dtype, epsilon, version, stream))


def qk_norm_rope_cache(args: QkCacheArgs, stream=0) -> None:
    """Generalised Q/K norm + RoPE + cache store (sm120n_qk_norm_rope_cache)."""
    _check(load().sm120n_qk_norm_rope_cache(ctypes.byref(args), stream))


def rms_norm_fp8_quant(input_ptr, residual_ptr, weight_ptr, residual_output_ptr, output_ptr,
                       scale_ptr, token_scales_ptr, scale_ub_ptr, rows, hidden_size, dtype,
                       epsilon=1e-6, stream=0) -> None:
    """RMSNorm (+ residual add) with fp8 e4m3 output; pass 0 / None for absent
    pointers (sm120n_rms_norm_fp8_quant)."""
    _check(load().sm120n_rms_norm_fp8_quant(
        input_ptr, residual_ptr, weight_ptr, residual_output_ptr, output_ptr, scale_ptr,
        token_scales_ptr, scale_ub_ptr, rows, hidden_size, dtype, epsilon, stream))


def rms_norm_fp4_quant(input_ptr, residual_ptr, weight_ptr, residual_output_ptr, output_ptr,
                       block_scales_ptr, global_scale_ptr, rows, hidden_size, dtype,
                       epsilon=1e-6, scale_layout=SCALES_TILED_128X4, stream=0) -> None:
    """RMSNorm (+ residual add) with NVFP4 output and e4m3 block scales; pass
    0 / None for an absent residual (sm120n_rms_norm_fp4_quant)."""
    _check(load().sm120n_rms_norm_fp4_quant(
        input_ptr, residual_ptr, weight_ptr, residual_output_ptr, output_ptr, block_scales_ptr,
        global_scale_ptr, rows, hidden_size, dtype, epsilon, scale_layout, stream))


def qkv_proj_norm_rope_cache(hidden_ptr, qkv_weight_ptr, qkv_ptr, tokens, hidden_size,
                             query_heads, key_heads, query_weight_ptr=None, key_weight_ptr=None,
                             positions_ptr=None, cos_sin_ptr=None, rope_positions=0,
                             key_cache_ptr=None, value_cache_ptr=None, slot_mapping_ptr=None,
                             cache_slots=0, epsilon=1e-6, epilogue=1, stream=0) -> None:
    """QKV projection on the tensor cores with the Q/K norm + RoPE + KV store
    in its epilogue (epilogue=1) or as a plain GEMM (epilogue=0)
    (sm120n_qkv_proj_norm_rope_cache)."""
    _check(load().sm120n_qkv_proj_norm_rope_cache(
        hidden_ptr, qkv_weight_ptr, qkv_ptr, tokens, hidden_size, query_heads, key_heads,
        query_weight_ptr, key_weight_ptr, positions_ptr, cos_sin_ptr, rope_positions,
        key_cache_ptr, value_cache_ptr, slot_mapping_ptr, cache_slots, epsilon, epilogue,
        stream))
