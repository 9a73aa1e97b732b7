"""Parity metrics and golden-fixture loading shared by the tests.

Tolerances (the bar every parity test states):
  * norm outputs (RMSNorm, fused add + RMSNorm): at most 1 ulp of the storage
    dtype for bf16 / fp16, at most 4 ulp for fp32, measured as the distance
    between the two values on the dtype's ordered bit lattice. Residual
    outputs (round(x + r)) must be bit-exact.
  * RoPE outputs: the norm-stage bar -- k ulp on t = round(x * inv_rms), the
    first rounding -- propagated exactly through the later roundings:
      |dn| <= k * (ulp(t)|w| + ulp(n))           n = round(t * w)
      |dy| <= |dn_i||c_i| + |dn_j||s_i| + k * ulp(y)
    k = 1 for bf16 / fp16 and 4 for fp32; each ulp is taken at the larger of
    the exact and the rounded magnitude. The first term matters: the fp32
    sum of squares may end one ulp apart in a different (equally valid)
    summation order, which flips the first rounding of a few elements per
    million, and the weight multiply can carry that flip into 2 ulp of n
    when t * w crosses a binade. Near-zero outputs come from cancellation,
    so an ulp of the output alone is not a meaningful bar.
  * KV-cache slots: bit-exact.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import math

import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
NAMES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}
MANTISSA_BITS = {torch.float32: 23, torch.float16: 10, torch.bfloat16: 7}
MIN_EXPONENT = {torch.float32: -126, torch.float16: -14, torch.bfloat16: -126}


def ordered(t: torch.Tensor) -> torch.Tensor:
    """Map floats to int64 so that adjacent representable values differ by 1."""
    if t.dtype == torch.float32:
        bits = t.contiguous().view(torch.int32).to(torch.int64)
        mag = bits & 0x7FFFFFFF
        return torch.where(bits < 0, -mag, mag)
    bits = t.contiguous().view(torch.int16).to(torch.int64) & 0xFFFF
    mag = bits & 0x7FFF
    return torch.where(bits >= 0x8000, -mag, mag)


def ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    assert a.dtype == b.dtype and a.shape == b.shape, (a.dtype, b.dtype, a.shape, b.shape)
    return (ordered(a.cpu()) - ordered(b.cpu())).abs()


def ulp_at(magnitude: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Spacing of `dtype` values at |magnitude| (float64)."""
    m = magnitude.abs().to(torch.float64)
    exponent = torch.floor(torch.log2(torch.clamp(m, min=1e-300)))
    exponent = torch.clamp(exponent, min=MIN_EXPONENT[dtype])
    return torch.pow(2.0, exponent - MANTISSA_BITS[dtype])


def default_norm_ulps(dtype: torch.dtype, row_length: int = 1024) -> int:
    """Norm-output bar. 16-bit outputs: 1 ulp (the final rounding to the
    activation dtype absorbs the fp32 sum-order difference). fp32 outputs:
    4 ulp for rows of up to 1024 elements (the reference's fp32 workload), and
    for longer rows 4 * ceil(sqrt(n / 1024)): the kernels and the oracle add
    the n squares in different, equally valid fp32 orders, and the rounding
    error of a sum of n positive terms grows with sqrt(n) (a different order
    moves inv_rms, and so every output of the row, by that relative amount)."""
    if dtype != torch.float32:
        return 1
    return 4 * max(1, math.ceil(math.sqrt(row_length / 1024)))


def assert_ulp_close(actual: torch.Tensor, expected: torch.Tensor, max_ulp: int | None = None,
                     what: str = "") -> None:
    if max_ulp is None:
        max_ulp = default_norm_ulps(expected.dtype, expected.shape[-1] if expected.dim() else 1)
    d = ulp_distance(actual, expected)
    worst = int(d.max()) if d.numel() else 0
    if worst > max_ulp:
        idx = int(d.flatten().argmax())
        raise AssertionError(
            f"{what}: {int((d > max_ulp).sum())} of {d.numel()} elements differ by more than "
            f"{max_ulp} ulp (worst {worst} ulp at flat index {idx}: "
            f"{actual.flatten()[idx].item()} vs {expected.flatten()[idx].item()})")


def assert_bitwise_equal(actual: torch.Tensor, expected: torch.Tensor, what: str = "") -> None:
    a, e = actual.detach().cpu().contiguous(), expected.detach().cpu().contiguous()
    assert a.dtype == e.dtype and a.shape == e.shape, (what, a.dtype, e.dtype, a.shape, e.shape)
    view = torch.int32 if a.dtype == torch.float32 else torch.int16
    if a.dtype in (torch.int32, torch.int64):
        view = a.dtype
    mism = (a.view(view) != e.view(view))
    if bool(mism.any()):
        idx = int(mism.flatten().nonzero()[0])
        raise AssertionError(f"{what}: {int(mism.sum())} of {mism.numel()} elements differ "
                             f"bitwise (first at flat index {idx})")


def rope_bound(x: torch.Tensor, weight: torch.Tensor, positions: torch.Tensor,
               cos_sin: torch.Tensor, expected: torch.Tensor, k: int | None = None,
               eps: float = 1e-6, interleaved: bool = False) -> torch.Tensor:
    """Propagation part of the RoPE tolerance for a [T, H, D] head tensor
    (module docstring): |dn_i||c_i| + |dn_j||s_i| with
    |dn| = k * (ulp(t)|w| + ulp(n)), t and n evaluated in fp64 from the inputs.
    The rotary width R is cos_sin's last dimension (R <= D); elements beyond R
    are not rotated and get |dn|. Partners are (i, i + R/2), or (2i, 2i + 1)
    when `interleaved`. assert_rope_close / rope_violations add k ulp of the
    output."""
    dtype = expected.dtype
    k = default_rope_k(dtype) if k is None else k
    xd = x.detach().cpu().to(torch.float64)
    rotary = cos_sin.shape[-1]
    half = rotary // 2
    w = weight.detach().cpu().to(torch.float64)
    t = xd * torch.rsqrt(xd.square().mean(-1, keepdim=True) + eps)
    n = t * w

    def ulp_rounded(v):
        return torch.maximum(ulp_at(v, dtype), ulp_at(v.to(dtype).to(torch.float64), dtype))

    dn = k * (ulp_rounded(t) * w.abs() + ulp_rounded(n))
    rows = cos_sin.detach().cpu().reshape(-1, rotary).to(torch.float64)[positions.cpu().long()]
    c, s = rows[:, None, :half].abs(), rows[:, None, half:].abs()
    rot = dn[..., :rotary]
    if interleaved:
        d1, d2 = rot[..., 0::2], rot[..., 1::2]
        bound = torch.stack((d1 * c + d2 * s, d2 * c + d1 * s), dim=-1).flatten(-2)
    else:
        d1, d2 = rot[..., :half], rot[..., half:]
        bound = torch.cat((d1 * c + d2 * s, d2 * c + d1 * s), dim=-1)
    return torch.cat((bound, dn[..., rotary:]), dim=-1)


def default_rope_k(dtype: torch.dtype) -> int:
    return 4 if dtype == torch.float32 else 1


def rope_violations(actual: torch.Tensor, expected: torch.Tensor, bound: torch.Tensor,
                    k: int | None = None) -> torch.Tensor:
    """Mask of outputs outside `bound` + k ulp of the output (taken at the larger
    of the two magnitudes)."""
    k = default_rope_k(expected.dtype) if k is None else k
    a = actual.detach().cpu().to(torch.float64)
    e = expected.detach().cpu().to(torch.float64)
    out_ulp = ulp_at(torch.maximum(a.abs(), e.abs()), expected.dtype)
    return (a - e).abs() > bound + k * out_ulp


def assert_rope_close(actual: torch.Tensor, expected: torch.Tensor, bound: torch.Tensor,
                      what: str = "") -> None:
    bad = rope_violations(actual, expected, bound)
    if bool(bad.any()):
        a = actual.detach().cpu().to(torch.float64)
        e = expected.detach().cpu().to(torch.float64)
        idx = int(bad.flatten().nonzero()[0])
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {bad.numel()} RoPE outputs exceed the propagated "
            f"bound (first at flat index {idx}: {a.flatten()[idx].item()} vs "
            f"{e.flatten()[idx].item()}, propagation bound {bound.flatten()[idx].item()})")


def strict_rope_violations(actual: torch.Tensor, expected: torch.Tensor, normed: torch.Tensor,
                           positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """Mask of RoPE outputs outside the strict bar |dy| <= 1 ulp(max(|n_i c_i|,
    |n_j s_i|)) (output i of a half-split pair (i, j): y_i = n_i c_i - n_j s_i,
    y_j = n_j c_i + n_i s_i), ulps of the activation dtype. `normed` is the
    oracle's n = round(round(x * inv_rms) * w) for [T, H, D] heads. The
    propagated bar above is the one every output must meet; this stricter
    one is reported as a count, since a different fp32 summation order
    legitimately flips the first rounding of a few elements per million."""
    dtype = expected.dtype
    n = normed.detach().cpu().to(torch.float64)
    rotary = cos_sin.shape[-1]
    half = rotary // 2
    rows = cos_sin.detach().cpu().reshape(-1, rotary).to(torch.float64)[positions.cpu().long()]
    c, s = rows[:, None, :half], rows[:, None, half:]
    n1, n2 = n[..., :half], n[..., half:rotary]
    first = torch.maximum((n1 * c).abs(), (n2 * s).abs())
    second = torch.maximum((n2 * c).abs(), (n1 * s).abs())
    scale = torch.cat((first, second), dim=-1)
    a = actual.detach().cpu().to(torch.float64)[..., :rotary]
    e = expected.detach().cpu().to(torch.float64)[..., :rotary]
    return (a - e).abs() > ulp_at(scale, dtype)


def load_golden(name: str) -> dict:
    """Fixture `name` as a dict of CPU tensors (bf16 restored from raw bits)."""
    with np.load(GOLDEN / f"{name}.npz") as data:
        raw = {k: data[k] for k in data.files}
    dtype = NAMES[str(raw.pop("dtype"))]
    out = {"dtype": dtype}
    for key, arr in raw.items():
        if arr.dtype == np.uint16:
            out[key] = torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
        elif arr.ndim == 0:
            out[key] = arr.item()
        else:
            out[key] = torch.from_numpy(arr.copy())
    return out


def golden_names(prefix: str) -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob(f"{prefix}*.npz"))
