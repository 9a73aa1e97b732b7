"""The parity bar itself, checked on the CPU.

The kernels sum squares in a different fp32 order than the oracle (an 8-lane
FMA accumulation and a butterfly over lanes, as in csrc/head_norm_rope.cu).
This file restates that order in numpy and shows that the differences it
causes are exactly the ones the bar in numerics.py allows: inv_rms differs by
an ulp on a fraction of heads, the first bf16 rounding flips on a few
elements per million, and every Q/K output stays inside the propagated RoPE
bound.
"""
import numpy as np
import torch

from numerics import rope_bound, rope_violations


def bf16(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def kernel_order_sum(sq):
    """Lane p accumulates elements [8p, 8p+8) then [64+8p, 64+8p+8); lanes are
    then combined by xor-butterfly (offsets 4, 2, 1)."""
    v = np.zeros((sq.shape[0], 8), np.float32)
    for part in range(8):
        acc = np.zeros(sq.shape[0], np.float32)
        for i in list(range(8 * part, 8 * part + 8)) + list(range(64 + 8 * part, 72 + 8 * part)):
            acc = (acc + sq[:, i]).astype(np.float32)
        v[:, part] = acc
    for off in (4, 2, 1):
        v = (v + v[:, [p ^ off for p in range(8)]]).astype(np.float32)
    return v[:, 0]


def oracle_order_sum(sq):
    """16 lanes x 4 accumulators, then a pairwise tree (oracle/norm_oracle.c)."""
    acc = np.zeros((sq.shape[0], 4, 16), np.float32)
    for blk in range(sq.shape[1] // 64):
        for a in range(4):
            acc[:, a] = (acc[:, a] + sq[:, 64 * blk + 16 * a:64 * blk + 16 * a + 16]).astype(np.float32)
    lane = acc[:, 0]
    for a in range(1, 4):
        lane = (lane + acc[:, a]).astype(np.float32)
    for width in (8, 4, 2, 1):
        lane = lane.copy()
        lane[:, :width] = (lane[:, :width] + lane[:, width:2 * width]).astype(np.float32)
    return lane[:, 0]


def inv_rms(total):
    mean = (total * np.float32(1 / 128)).astype(np.float32)
    shifted = (mean + np.float32(1e-6)).astype(np.float32)
    return (np.float32(1) / np.sqrt(shifted.astype(np.float64)).astype(np.float32)).astype(np.float32)


def rotate(n, c, s):
    n1, n2 = n[:, :64], n[:, 64:]
    lo = ((n1 * c).astype(np.float32) - (n2 * s).astype(np.float32)).astype(np.float32)
    hi = ((n2 * c).astype(np.float32) + (n1 * s).astype(np.float32)).astype(np.float32)
    return bf16(np.concatenate([lo, hi], 1))


def test_summation_order_differences_stay_inside_the_bar():
    rng = np.random.default_rng(0)
    heads = 60000
    x = bf16(rng.standard_normal((heads, 128)).astype(np.float32))
    w = bf16((1 + 0.1 * rng.standard_normal(128)).astype(np.float32))
    sq = (x.astype(np.float64) ** 2).astype(np.float32)  # exact for bf16 inputs
    inv_k, inv_o = inv_rms(kernel_order_sum(sq)), inv_rms(oracle_order_sum(sq))
    assert 0.01 < np.mean(inv_k != inv_o) < 0.5          # the orders really differ
    n_k = bf16((bf16((x * inv_k[:, None]).astype(np.float32)) * w).astype(np.float32))
    n_o = bf16((bf16((x * inv_o[:, None]).astype(np.float32)) * w).astype(np.float32))
    inv_freq = (1.0 / (1e6 ** (np.arange(0, 128, 2, dtype=np.float32) / 128))).astype(np.float32)
    pos = rng.integers(0, 32768, heads)
    angles = (pos[:, None].astype(np.float32) * inv_freq[None]).astype(np.float32)
    cache = np.concatenate([np.cos(angles), np.sin(angles)], 1).astype(np.float32)
    c, s = cache[:, :64], cache[:, 64:]
    y_k, y_o = rotate(n_k, c, s), rotate(n_o, c, s)
    to_t = lambda a: torch.from_numpy(a).to(torch.bfloat16).view(heads, 1, 128)
    bound = rope_bound(to_t(x), torch.from_numpy(w).to(torch.bfloat16), torch.arange(heads),
                       torch.from_numpy(cache), to_t(y_o))
    assert int(rope_violations(to_t(y_k), to_t(y_o), bound).sum()) == 0
