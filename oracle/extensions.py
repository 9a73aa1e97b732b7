"""CPU oracle for the engine-side extensions (csrc/head_cache.cu,
csrc/norm_quant.cu).

TEST INFRASTRUCTURE. Only the test suite and ``bench.py``'s checks use this
module, as the checker; the shipped package never imports it.

The reference project has no counterpart for these operators, so the oracle
generalises its PyTorch oracle (``sm120_rmsnorm/reference.py:27-49`` for the
per-head norm + RoPE; ``:5-24`` for RMSNorm and the residual add), operation
for operation, along the extension axes:

* head sizes other than 128 and partial rotary: the norm covers all head_dim
  elements; RoPE the first ``rotary_dim`` (= ``cos_sin_cache.size(-1)``);
  the rest is the normalised, weighted value;
* interleaved pairs (2i, 2i + 1) next to the reference's half split;
* paged caches in NHD [blocks, block_size, Hk, D] or HND [blocks, Hk,
  block_size, D] order;
* fp8 e4m3fn storage: ``sat(v) = clamp(v, -448, 448)`` rounded to the nearest
  e4m3fn value, ties to even (PyTorch's float8_e4m3fn conversion after the
  clamp; pinned against :func:`e4m3_round_reference`, written from the format
  definition, by the CPU tests).

``rsqrt(mean(x^2) + eps)`` is evaluated in IEEE fp32 as ``1 / sqrt(.)`` with
a correctly rounded square root and divide (numpy), like the C oracle and the
kernels: PyTorch's vectorised CPU ``sqrt`` / ``rsqrt`` are not correctly
rounded on every build (on AVX-512 about 0.5% of results differ in the last
bit), so an oracle built on them would be reproducible only to one ulp.
With inputs whose sums of squares are exact in fp32, every operation here is
then defined to the bit.
"""
from __future__ import annotations

import numpy as np
import torch

FP8_MAX = 448.0
MIN_TOKEN_SCALE = np.float32(1.0) / np.float32(448.0 * 512.0)


# ---- fp8 e4m3fn ----------------------------------------------------------------
def fp8_e4m3(v: torch.Tensor) -> torch.Tensor:
    """sat(v) for an fp32 tensor, as float8_e4m3fn."""
    assert v.dtype == torch.float32
    return v.clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)


def e4m3_decode(code: int) -> float:
    """Value of an e4m3fn byte from the format definition: 1 sign bit, 4
    exponent bits (bias 7), 3 mantissa bits, subnormals at exponent 0, and
    S.1111.111 the only NaN (no infinities)."""
    sign = -1.0 if code & 0x80 else 1.0
    exponent = (code >> 3) & 0xF
    mantissa = code & 0x7
    if exponent == 0xF and mantissa == 0x7:
        return float("nan")
    if exponent == 0:
        return sign * mantissa * 2.0 ** -9
    return sign * (1.0 + mantissa / 8.0) * 2.0 ** (exponent - 7)


def e4m3_round_reference(values: np.ndarray) -> np.ndarray:
    """Bytes of sat(v) by exhaustive nearest-value search among the codes of
    v's sign (so -0.0 and small negatives round to -0), ties to the even
    code (the even mantissa), independent of PyTorch's conversion. For
    pinning only."""
    table = np.array([e4m3_decode(c) for c in range(256)])
    out = np.empty(values.shape, dtype=np.uint8)
    flat, res = np.clip(values.astype(np.float64).reshape(-1), -FP8_MAX, FP8_MAX), out.reshape(-1)
    for i, x in enumerate(flat):
        codes = np.arange(0x80, 0xFF) if np.signbit(x) else np.arange(0x00, 0x7F)
        dist = np.abs(table[codes] - x)
        ties = codes[dist == dist.min()]
        res[i] = int(ties[0] if len(ties) == 1 else ties[(ties & 1) == 0][0])
    return out


# ---- inverse RMS ------------------------------------------------------------------
def inv_rms(xf: torch.Tensor, eps: float) -> torch.Tensor:
    """1 / sqrt(mean(x^2) + eps) over the last dimension of an fp32 tensor,
    every step rounded once (IEEE fp32); keepdim."""
    mean = xf.square().mean(dim=-1, keepdim=True).numpy()  # sum / n
    shifted = mean + np.float32(eps)
    return torch.from_numpy(np.float32(1.0) / np.sqrt(shifted))


# ---- generalised Q/K norm + RoPE + cache store -----------------------------------
def _norm_then_rope(x, weight, rows, rotary_dim, is_neox, eps):
    """reference.py:35-48 generalised: [T, H, D] -> [T, H, D]."""
    dtype = x.dtype
    xf = x.float()
    normalized = (xf * inv_rms(xf, eps)).to(dtype)  # F.rms_norm(x.float(), (D,), None, eps)
    normalized = normalized * weight
    half = rotary_dim // 2
    cos, sin = rows[:, None, :half], rows[:, None, half:]
    rotating = normalized[..., :rotary_dim].float()
    if is_neox:
        first, second = rotating.chunk(2, dim=-1)
    else:
        first, second = rotating[..., 0::2], rotating[..., 1::2]
    rotated_first = first * cos - second * sin
    rotated_second = second * cos + first * sin
    if is_neox:
        rotated = torch.cat((rotated_first, rotated_second), dim=-1)
    else:
        rotated = torch.stack((rotated_first, rotated_second), dim=-1).flatten(-2)
    return torch.cat((rotated.to(dtype), normalized[..., rotary_dim:]), dim=-1)


def qk_norm_rope_cache(query, key, value, query_weight, key_weight, positions, cos_sin_cache,
                       key_cache=None, value_cache=None, slot_mapping=None, k_scale=None,
                       v_scale=None, is_neox=True, kv_cache_layout="NHD", eps=1e-6):
    """Expected (query, key, key_cache, value_cache) after the operator, as new
    CPU tensors (caches None without a store). Tokens whose position lies
    outside the cos/sin cache are unchanged and store nothing; slots outside
    the cache store nothing."""
    q, k = query.cpu().clone(), key.cpu().clone()
    table = cos_sin_cache.cpu().float()
    rotary_dim = table.size(-1)
    table = table.reshape(-1, rotary_dim)
    pos = positions.cpu().long()
    valid = (pos >= 0) & (pos < table.size(0))
    rows = table[pos.clamp(0, max(table.size(0) - 1, 0))]
    qw, kw = query_weight.cpu(), key_weight.cpu()
    if q.numel():
        q[valid] = _norm_then_rope(q, qw, rows, rotary_dim, is_neox, eps)[valid]
    if k.numel():
        k[valid] = _norm_then_rope(k, kw, rows, rotary_dim, is_neox, eps)[valid]
    if key_cache is None:
        return q, k, None, None
    kc, vc = key_cache.cpu().clone(), value_cache.cpu().clone()
    v = value.cpu()
    nhd = kv_cache_layout == "NHD"
    block_size = kc.size(1) if nhd else kc.size(2)
    capacity = kc.size(0) * block_size
    fp8 = kc.dtype in (torch.float8_e4m3fn, torch.uint8)
    for t, slot in enumerate(slot_mapping.cpu().tolist()):
        if not bool(valid[t]) or slot < 0 or slot >= capacity:
            continue
        block, offset = divmod(slot, block_size)
        kt, vt = k[t], v[t]
        if fp8:
            kt = fp8_e4m3(kt.float() / k_scale.cpu().float().reshape(()))
            vt = fp8_e4m3(vt.float() / v_scale.cpu().float().reshape(()))
            if kc.dtype == torch.uint8:
                kt, vt = kt.view(torch.uint8), vt.view(torch.uint8)
        if nhd:
            kc[block, offset], vc[block, offset] = kt, vt
        else:
            kc[block, :, offset], vc[block, :, offset] = kt, vt
    return q, k, kc, vc


# ---- RMSNorm with fp8 quantisation ------------------------------------------------
def rms_norm_rows(x, weight, eps=1e-6, residual=None):
    """(y, residual_out): reference.py:5-24 (RMSNorm of x, or of round(x + r))."""
    x = x.cpu()
    s = x + residual.cpu() if residual is not None else x
    sf = s.float()
    y = (sf * inv_rms(sf, eps) * weight.cpu().float()).to(x.dtype)
    return y, (s if residual is not None else None)


def quantise_rows(y, scale=None, scale_ub=None):
    """(q, token_scales) for a normalised row tensor y: static with a
    one-element ``scale``, dynamic per row otherwise."""
    yf = y.float()
    if scale is not None:
        inv = torch.reciprocal(scale.cpu().float().reshape(()))
        return fp8_e4m3(yf * inv), None
    peak = yf.abs().amax(dim=-1)
    if scale_ub is not None:
        peak = torch.minimum(peak, scale_ub.cpu().float().reshape(()))
    token_scales = torch.maximum(peak / FP8_MAX, torch.tensor(MIN_TOKEN_SCALE))
    return fp8_e4m3(yf * torch.reciprocal(token_scales)[..., None]), token_scales


def rms_norm_fp8_quant(x, weight, eps=1e-6, residual=None, scale=None, scale_ub=None):
    """(q, token_scales, residual_out) of the norm + quantisation operators."""
    y, residual_out = rms_norm_rows(x, weight, eps, residual)
    q, token_scales = quantise_rows(y, scale, scale_ub)
    return q, token_scales, residual_out


# ---- NVFP4 (e2m1 values, e4m3 block scales) -----------------------------------------
E2M1_MAGNITUDES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float64)


def e2m1_codes(values: np.ndarray) -> np.ndarray:
    """4-bit e2m1 codes of fp32 values from the format definition (1 sign bit,
    2 exponent bits, 1 mantissa bit; magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6):
    nearest magnitude, ties to the even code, saturating at 6, sign kept (so
    small negatives give -0, code 8)."""
    v = values.astype(np.float64)
    mag = np.minimum(np.abs(v), 6.0)
    dist = np.abs(mag[..., None] - E2M1_MAGNITUDES)
    best = dist.min(axis=-1, keepdims=True)
    ties = dist == best
    # among tied magnitudes prefer the even code
    even = ties & (np.arange(8) % 2 == 0)
    choice = np.where(even.any(axis=-1, keepdims=True), even, ties)
    code = np.argmax(choice, axis=-1).astype(np.uint8)
    return np.where(np.signbit(v), code | 8, code).astype(np.uint8)


def nvfp4_scale_offsets(rows: int, blocks: int, tiled: bool) -> np.ndarray:
    """Byte offset of scale (row m, block k) in the row-major or the 128 x 4
    tiled layout ([rows, blocks] array of offsets)."""
    m = np.arange(rows)[:, None]
    k = np.arange(blocks)[None, :]
    if not tiled:
        return m * blocks + k
    columns = (blocks + 3) // 4 * 4
    tile = (m // 128) * (columns // 4) + k // 4
    return tile * 512 + ((m % 32) * 4 + (m % 128) // 32) * 4 + k % 4


def nvfp4_quantise(y: torch.Tensor, global_scale: float, tiled: bool):
    """(packed [rows, hidden / 2] uint8, scale bytes) of a normalised row
    tensor y; the scale buffer is sized for the layout, padding zero."""
    yf = y.float().reshape(-1, y.shape[-1]).numpy()
    rows, hidden = yf.shape
    blocks = hidden // 16
    g = np.float32(global_scale)
    peak = np.abs(yf.reshape(rows, blocks, 16)).max(axis=-1)
    one_sixth = np.float32(1.0) / np.float32(6.0)
    wanted = (g * (peak * one_sixth).astype(np.float32)).astype(np.float32)
    codes = fp8_e4m3(torch.from_numpy(wanted)).view(torch.uint8).numpy()
    s = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    with np.errstate(divide="ignore"):
        r = np.where(s == 0, np.float32(0.0), g / np.where(s == 0, np.float32(1), s)).astype(np.float32)
    v = (yf.reshape(rows, blocks, 16) * r[..., None]).astype(np.float32).reshape(rows, hidden)
    q = e2m1_codes(v)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    if tiled:
        size = (rows + 127) // 128 * 128 * ((blocks + 3) // 4 * 4)
    else:
        size = rows * blocks
    scales = np.zeros(size, dtype=np.uint8)
    scales[nvfp4_scale_offsets(rows, blocks, tiled)] = codes
    return torch.from_numpy(packed), torch.from_numpy(scales)


def rms_norm_nvfp4_quant(x, weight, global_scale, eps=1e-6, residual=None, tiled=True):
    """(packed, scales, residual_out) of the NVFP4 norm operator."""
    y, residual_out = rms_norm_rows(x, weight, eps, residual)
    packed, scales = nvfp4_quantise(y, global_scale, tiled)
    return packed, scales, residual_out
