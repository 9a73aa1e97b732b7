"""CPU oracle loader: builds and binds ``norm_oracle.c``.

TEST INFRASTRUCTURE. Only the test suite, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` use this module, as the checker (or the timed
CPU baseline). The shipped package never imports it.

The C file restates the reference's PyTorch oracle
(``sm120_rmsnorm/reference.py`` in the reference project); the functions
below take contiguous CPU tensors and call it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "norm_oracle.c"
BUILD_DIR = HERE / "_build"
LIBRARY = BUILD_DIR / "libnorm_oracle.so"

F32, F16, BF16 = 0, 1, 2
DTYPE_CODES = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

# x86-64-v3 (AVX2) keeps the CPU baseline vectorised on any current server
# CPU; -ffp-contract=off keeps every product and sum separately rounded.
CFLAGS = [
    "-O3", "-march=x86-64-v3", "-fPIC", "-shared", "-fopenmp",
    "-ffp-contract=off", "-fno-fast-math", "-std=gnu11",
]

_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle into ``oracle/_build`` (skipped when up to date)."""
    BUILD_DIR.mkdir(exist_ok=True)
    if (not force and LIBRARY.exists()
            and LIBRARY.stat().st_mtime >= SOURCE.stat().st_mtime):
        return LIBRARY
    tmp = LIBRARY.with_suffix(f".so.tmp{os.getpid()}")
    subprocess.run(["gcc", *CFLAGS, str(SOURCE), "-o", str(tmp), "-lm"],
                   check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            path = LIBRARY if LIBRARY.exists() else build()
            handle = ctypes.CDLL(str(path))
            i64, vp, i32, f32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_float
            handle.oracle_rms_norm.argtypes = [vp, vp, vp, i64, i64, i32, f32]
            handle.oracle_fused_add_rms_norm.argtypes = [vp, vp, vp, vp, vp, i64, i64, i32, f32]
            handle.oracle_qk_rms_norm_rope.argtypes = [
                vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, f32]
            handle.oracle_qk_rms_norm_rope_kv.argtypes = [
                vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                i64, i64, i64, i64, i64, i64, i32, f32]
            handle.oracle_set_threads.argtypes = [i32]
            handle.oracle_get_threads.restype = i32
            _lib = handle
    return _lib


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def get_threads() -> int:
    return int(lib().oracle_get_threads())


def _cpu(t: torch.Tensor) -> torch.Tensor:
    if t.device.type != "cpu" or not t.is_contiguous():
        raise ValueError("oracle functions take contiguous CPU tensors")
    return t


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else _cpu(t).data_ptr()


def _check(rc: int, name: str) -> None:
    if rc != 0:
        raise ValueError(f"{name}: invalid arguments")


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """reference.py:5-11 on CPU; returns a new tensor."""
    out = torch.empty_like(x)
    hidden = x.shape[-1]
    _check(lib().oracle_rms_norm(_ptr(x), _ptr(weight), _ptr(out), x.numel() // hidden,
                                 hidden, DTYPE_CODES[x.dtype], eps), "rms_norm")
    return out


def fused_add_rms_norm_out(x, residual, weight, out, residual_out, eps: float = 1e-6) -> None:
    """reference.py:14-24 into caller buffers (out may be x, residual_out may be residual)."""
    hidden = x.shape[-1]
    _check(lib().oracle_fused_add_rms_norm(
        _ptr(x), _ptr(residual), _ptr(weight), _ptr(out), _ptr(residual_out),
        x.numel() // hidden, hidden, DTYPE_CODES[x.dtype], eps), "fused_add_rms_norm")


def fused_add_rms_norm(x, residual, weight, eps: float = 1e-6):
    """Returns (output, residual_output) like reference.py:14-24."""
    out, res = torch.empty_like(x), torch.empty_like(x)
    fused_add_rms_norm_out(x, residual, weight, out, res, eps)
    return out, res


def qk_rms_norm_rope_(query, key, query_weight, key_weight, positions, cos_sin_cache,
                      eps: float = 1e-6) -> None:
    """reference.py:27-49, in place on query and key."""
    head_dim = query.shape[-1]
    _check(lib().oracle_qk_rms_norm_rope(
        _ptr(query), _ptr(key), _ptr(query_weight), _ptr(key_weight), _ptr(positions),
        _ptr(cos_sin_cache), query.shape[0], query.shape[1], key.shape[1], head_dim,
        cos_sin_cache.numel() // head_dim, DTYPE_CODES[query.dtype], eps), "qk_rms_norm_rope")


def qk_rms_norm_rope_kv_(query, key, value, query_weight, key_weight, positions,
                         cos_sin_cache, key_cache, value_cache, slot_mapping,
                         eps: float = 1e-6) -> None:
    """reference.py:27-49 plus the paged KV store of csrc/rmsnorm_kernels.cu:425-435."""
    head_dim = query.shape[-1]
    key_heads = key.shape[1]
    _check(lib().oracle_qk_rms_norm_rope_kv(
        _ptr(query), _ptr(key), _ptr(value), _ptr(query_weight), _ptr(key_weight),
        _ptr(positions), _ptr(cos_sin_cache), _ptr(key_cache), _ptr(value_cache),
        _ptr(slot_mapping), query.shape[0], query.shape[1], key_heads, head_dim,
        cos_sin_cache.numel() // head_dim, key_cache.numel() // (key_heads * head_dim),
        DTYPE_CODES[query.dtype], eps), "qk_rms_norm_rope_kv")
