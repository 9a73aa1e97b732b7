"""Q/K RoPE outputs of every Q/K workload configuration against the strict
bar |dy| <= 1 ulp(max(|n_i c_i|, |n_j s_i|)) (n: the oracle's normalised,
weighted head; (c, s): the position's cos / sin). Every output must meet the
propagated bar of numerics.py; the number of outputs outside the strict bar
is printed and must stay at or below 1e-5 of the outputs (rounded up). A
different fp32 summation order than the oracle's flips the first rounding of
a few elements per million, which the strict bar counts and the propagated
bar covers, so a regression of any size shows up here as a count.

KV-cache slots are checked bit for bit: the key slot holds exactly the kernel's
rotated K and the value slot the input V."""
import math

import pytest
import torch

from gpu_cases import assert_bitwise_equal, check_rope, expect_qk, expect_qk_kv
from numerics import strict_rope_violations
from sm120_rmsnorm import fused_qk_rms_norm_rope, fused_qk_rms_norm_rope_kv

pytestmark = pytest.mark.gpu


def rope_cache(positions: int) -> torch.Tensor:
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
    f = torch.outer(torch.arange(positions, dtype=torch.float32, device="cuda"), inv)
    return torch.cat((f.cos(), f.sin()), dim=-1)


def _check_strict(got, want, x_in, w, pos, cache, what):
    # the oracle's n = round(round(x * inv) * w): RoPE at position 0 (cos 1, sin 0)
    zero = torch.zeros_like(pos)
    normed, _ = expect_qk(x_in, x_in[:, :1], w, w, zero, cache)
    check_rope(got, want, x_in, w, pos, cache, what=what)
    bad = strict_rope_violations(got, want, normed, pos, cache)
    count, total = int(bad.sum()), bad.numel()
    print(f"{what}: {count} of {total} outputs outside the 1-ulp bar ({count / total:.2e})")
    assert count <= math.ceil(1e-5 * total), f"{what}: {count} of {total} outside the 1-ulp bar"
    return count


CONFIGS = [  # (name, tokens, query heads, key heads, paged blocks, decode)
    ("decode B=1 16/8", 1, 16, 8, 2048, True),
    ("decode B=64 32/8", 64, 32, 8, 65536, True),
    ("decode B=256 32/8", 256, 32, 8, 65536, True),
    ("decode B=1024 32/8", 1024, 32, 8, 65536, True),
    ("prefill 32768 64/8", 32768, 64, 8, 2048, False),
]


@pytest.mark.parametrize("name,tokens,hq,hk,blocks,decode", CONFIGS, ids=[c[0] for c in CONFIGS])
def test_qk_kv_workload_strict_bar(name, tokens, hq, hk, blocks, decode):
    g = torch.Generator(device="cuda").manual_seed(tokens + 17)
    cpu_g = torch.Generator().manual_seed(tokens)
    bf = torch.bfloat16
    q = torch.randn(tokens, hq, 128, device="cuda", generator=g).to(bf)
    k = torch.randn(tokens, hk, 128, device="cuda", generator=g).to(bf)
    v = torch.randn(tokens, hk, 128, device="cuda", generator=g).to(bf)
    qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
    kw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
    cache = rope_cache(32768)
    if decode:
        pos = torch.randperm(32768, generator=cpu_g)[:tokens].cuda()
        slots = torch.randperm(blocks * 16, generator=cpu_g)[:tokens].to(torch.int32).cuda()
    else:
        pos = torch.arange(tokens, device="cuda")
        slots = torch.arange(tokens, device="cuda", dtype=torch.int32)
    kc = torch.zeros(blocks, 16, hk, 128, device="cuda", dtype=bf)
    vc = torch.zeros_like(kc)
    q_in, k_in = q.clone(), k.clone()
    fused_qk_rms_norm_rope_kv(q, k, v, qw, kw, pos, cache, kc, vc, slots)
    torch.cuda.synchronize()
    # the oracle on every token, or on a seeded sample of the prefill's
    rows = torch.arange(tokens) if tokens <= 1024 else \
        torch.randperm(tokens, generator=cpu_g)[:1024].sort().values
    rows_d = rows.cuda()
    sq, sk, sv, sp, ss = (t[rows_d] for t in (q_in, k_in, v, pos, slots))
    flat_k, flat_v = kc.view(-1, hk, 128), vc.view(-1, hk, 128)
    small_kc = torch.zeros(len(rows), 1, hk, 128, dtype=bf)
    want_q, want_k, want_kc, want_vc = expect_qk_kv(
        sq, sk, sv, qw, kw, sp, cache, small_kc, small_kc.clone(),
        torch.arange(len(rows), dtype=torch.int32))
    _check_strict(q[rows_d].cpu(), want_q, sq, qw, sp, cache, f"{name} query")
    _check_strict(k[rows_d].cpu(), want_k, sk, kw, sp, cache, f"{name} key")
    # the cache holds exactly the rotated K this kernel wrote and the input V
    assert_bitwise_equal(flat_k[ss.long()], k[rows_d], what=f"{name} key cache")
    assert_bitwise_equal(flat_v[ss.long()], sv, what=f"{name} value cache")
    assert_bitwise_equal(want_vc.view(-1, hk, 128), sv, what=f"{name} oracle value cache")


@pytest.mark.parametrize("tokens", [1, 4, 16, 64, 256])
def test_qk_no_kv_strict_bar(tokens):
    """fused_qk_rms_norm_rope at the reference benchmark's shapes (16 / 8
    heads, positions 0..T-1)."""
    g = torch.Generator(device="cuda").manual_seed(tokens + 29)
    bf = torch.bfloat16
    q = torch.randn(tokens, 16, 128, device="cuda", generator=g).to(bf)
    k = torch.randn(tokens, 8, 128, device="cuda", generator=g).to(bf)
    qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
    kw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
    pos = torch.arange(tokens, device="cuda")
    cache = rope_cache(32768)
    want_q, want_k = expect_qk(q, k, qw, kw, pos, cache)
    q_in, k_in = q.clone(), k.clone()
    fused_qk_rms_norm_rope(q, k, qw, kw, pos, cache)
    _check_strict(q.cpu(), want_q, q_in, qw, pos, cache, f"T={tokens} query")
    _check_strict(k.cpu(), want_k, k_in, kw, pos, cache, f"T={tokens} key")
