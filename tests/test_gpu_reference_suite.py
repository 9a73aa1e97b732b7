"""The reference's own correctness suite (tests/test_correctness.py in the
reference project, 180 cases), run against the B200 kernels.

Same operators, shapes, seeds, versions and weight distributions as the
reference file; the bar is tighter than its atol/rtol: every output is
compared with the oracle at the ulp tolerances stated in numerics.py
(1 ulp for bf16 / fp16 norm outputs, bit-exact residuals and KV slots,
propagated-ulp bound for RoPE outputs).
"""
import pytest
import torch

from gpu_cases import (assert_bitwise_equal, check_norm, check_rope, expect_fused_add,
                       expect_qk, expect_qk_kv, expect_rms_norm)
from sm120_rmsnorm import (fused_add_rms_norm, fused_add_rms_norm_inplace,
                           fused_qk_rms_norm_rope, fused_qk_rms_norm_rope_kv, rms_norm)

pytestmark = pytest.mark.gpu
DTYPES = [torch.float16, torch.bfloat16, torch.float32]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", [(1, 1024), (17, 1024), (8, 768), (3, 1000), (2, 4, 2048)])
@pytest.mark.parametrize("version", [1, 2])
def test_rms_norm(dtype, shape, version):
    torch.manual_seed(7)
    x = torch.randn(shape, device="cuda", dtype=dtype)
    weight = torch.randn(shape[-1], device="cuda", dtype=dtype)
    actual = rms_norm(x, weight, version=version)
    check_norm(actual.cpu(), expect_rms_norm(x, weight), what=f"rms {shape}")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tokens", [1, 7, 64])
@pytest.mark.parametrize("version", [0, 2, 3, 4])
def test_fused_add_rms_norm(dtype, tokens, version):
    torch.manual_seed(11)
    x = torch.randn((tokens, 1024), device="cuda", dtype=dtype)
    residual = torch.randn_like(x)
    weight = torch.randn(1024, device="cuda", dtype=dtype)
    expected, expected_residual = expect_fused_add(x, residual, weight)
    actual, actual_residual = fused_add_rms_norm(x, residual, weight, version=version)
    assert_bitwise_equal(actual_residual, expected_residual, what="residual")
    check_norm(actual.cpu(), expected, what="output")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tokens", [1, 7, 64])
@pytest.mark.parametrize("version", [0, 2, 3, 4])
def test_fused_add_rms_norm_inplace(dtype, tokens, version):
    torch.manual_seed(13)
    x = torch.randn((tokens, 1024), device="cuda", dtype=dtype)
    residual = torch.randn_like(x)
    weight = torch.randn(1024, device="cuda", dtype=dtype)
    expected, expected_residual = expect_fused_add(x, residual, weight)
    fused_add_rms_norm_inplace(x, residual, weight, version=version)
    assert_bitwise_equal(residual, expected_residual, what="residual")
    check_norm(x.cpu(), expected, what="output")


@pytest.mark.parametrize("version", [3, 4])
def test_specialized_versions_reject_non_1024_hidden_size(version):
    x = torch.randn((4, 768), device="cuda", dtype=torch.float16)
    residual = torch.randn_like(x)
    weight = torch.randn(768, device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="hidden_size=1024"):
        fused_add_rms_norm(x, residual, weight, version=version)


def test_auto_dispatch_falls_back_for_generic_hidden_size():
    torch.manual_seed(17)
    x = torch.randn((5, 768), device="cuda", dtype=torch.float16)
    residual = torch.randn_like(x)
    weight = torch.randn(768, device="cuda", dtype=torch.float16)
    expected, expected_residual = expect_fused_add(x, residual, weight)
    actual, actual_residual = fused_add_rms_norm(x, residual, weight, version=0)
    assert_bitwise_equal(actual_residual, expected_residual, what="residual")
    check_norm(actual.cpu(), expected, what="output")


def make_rope_cache(max_position: int = 512, base: float = 1_000_000.0) -> torch.Tensor:
    """[P, 1, 128] fp32 cos || sin, as the reference tests build it."""
    inv_freq = 1.0 / (base ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
    freqs = torch.outer(torch.arange(max_position, dtype=torch.float32, device="cuda"), inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze(1)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tokens", [1, 7, 64])
@pytest.mark.parametrize("heads", [(16, 8), (8, 8), (4, 2)])
@pytest.mark.parametrize("version", [1, 2])
def test_fused_qk_rms_norm_rope(dtype, tokens, heads, version):
    torch.manual_seed(29)
    hq, hk = heads
    query = torch.randn((tokens, hq, 128), device="cuda", dtype=dtype)
    key = torch.randn((tokens, hk, 128), device="cuda", dtype=dtype)
    qw = torch.randn(128, device="cuda", dtype=dtype)
    kw = torch.randn(128, device="cuda", dtype=dtype)
    positions = torch.arange(tokens, device="cuda", dtype=torch.int64) * 3
    cache = make_rope_cache(max_position=max(tokens * 3, 1) + 1)
    q0, k0 = query.clone(), key.clone()
    eq, ek = expect_qk(query, key, qw, kw, positions, cache)
    fused_qk_rms_norm_rope(query, key, qw, kw, positions, cache, version=version)
    check_rope(query.cpu(), eq, q0, qw, positions, cache, what="query")
    check_rope(key.cpu(), ek, k0, kw, positions, cache, what="key")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_qk_rms_norm_rope_zero_input(dtype):
    query = torch.zeros((2, 16, 128), device="cuda", dtype=dtype)
    key = torch.zeros((2, 8, 128), device="cuda", dtype=dtype)
    weight = torch.ones(128, device="cuda", dtype=dtype)
    positions = torch.tensor([0, 511], device="cuda", dtype=torch.int64)
    fused_qk_rms_norm_rope(query, key, weight, weight, positions, make_rope_cache())
    assert not query.any() and not key.any()


def test_fused_qk_rms_norm_rope_rejects_other_head_dim():
    query = torch.randn((1, 16, 64), device="cuda", dtype=torch.float16)
    key = torch.randn((1, 8, 64), device="cuda", dtype=torch.float16)
    weight = torch.ones(64, device="cuda", dtype=torch.float16)
    positions = torch.zeros(1, device="cuda", dtype=torch.int64)
    cache = torch.zeros((1, 1, 64), device="cuda", dtype=torch.float32)
    with pytest.raises(RuntimeError, match="head_dim=128"):
        fused_qk_rms_norm_rope(query, key, weight, weight, positions, cache)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tokens", [1, 7, 64])
@pytest.mark.parametrize("version", [1, 4])
def test_fused_qk_rms_norm_rope_kv(dtype, tokens, version):
    torch.manual_seed(37)
    query = torch.randn((tokens, 16, 128), device="cuda", dtype=dtype)
    key = torch.randn((tokens, 8, 128), device="cuda", dtype=dtype)
    value = torch.randn_like(key)
    qw = torch.randn(128, device="cuda", dtype=dtype)
    kw = torch.randn(128, device="cuda", dtype=dtype)
    positions = torch.arange(tokens, device="cuda", dtype=torch.int64) * 2
    cache = make_rope_cache(max_position=max(tokens * 2, 1) + 1)
    slots = torch.arange(tokens, device="cuda", dtype=torch.int32) * 2
    if tokens > 1:
        slots[1] = -1
    key_cache = torch.randn((tokens * 2, 8, 128), device="cuda", dtype=dtype)
    value_cache = torch.randn_like(key_cache)
    q0, k0 = query.clone(), key.clone()
    eq, ek, ekc, evc = expect_qk_kv(query, key, value, qw, kw, positions, cache, key_cache,
                                    value_cache, slots)
    untouched_k, untouched_v = key_cache.clone(), value_cache.clone()
    fused_qk_rms_norm_rope_kv(query, key, value, qw, kw, positions, cache, key_cache,
                              value_cache, slots, version=version)
    check_rope(query.cpu(), eq, q0, qw, positions, cache, what="query")
    check_rope(key.cpu(), ek, k0, kw, positions, cache, what="key")
    # KV slots: the kernel's own rotated K and the input V, bit for bit;
    # every other slot (including the padded token's) unchanged.
    valid = slots >= 0
    untouched_k[slots[valid].long()] = key[valid]
    untouched_v[slots[valid].long()] = value[valid]
    assert_bitwise_equal(key_cache, untouched_k, what="key_cache")
    assert_bitwise_equal(value_cache, untouched_v, what="value_cache")
    assert_bitwise_equal(value_cache.cpu(), evc, what="value_cache vs oracle")
