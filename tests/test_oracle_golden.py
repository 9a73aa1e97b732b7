"""Pin the C oracle to vectors produced by the reference's own PyTorch oracle.

CPU only. The golden fixtures were made by tests/golden/make_golden.py from
the reference's sm120_rmsnorm/reference.py.
"""
import pytest
import torch

from numerics import (assert_bitwise_equal, assert_rope_close, assert_ulp_close,
                      golden_names, load_golden, rope_bound)
from oracle import oracle


@pytest.fixture(scope="module", autouse=True)
def _built():
    oracle.build()
    oracle.set_threads(2)


@pytest.mark.parametrize("name", golden_names("rms_"))
def test_rms_norm_matches_reference(name):
    g = load_golden(name)
    out = oracle.rms_norm(g["x"], g["w"], g["eps"])
    assert_ulp_close(out, g["out"], what=name)


@pytest.mark.parametrize("name", golden_names("fused_"))
def test_fused_add_rms_norm_matches_reference(name):
    g = load_golden(name)
    out, res = oracle.fused_add_rms_norm(g["x"], g["r"], g["w"], g["eps"])
    assert_bitwise_equal(res, g["res"], what=name + " residual")
    assert_ulp_close(out, g["out"], what=name)


@pytest.mark.parametrize("name", golden_names("fused_"))
def test_fused_add_rms_norm_in_place_aliasing(name):
    g = load_golden(name)
    x, r = g["x"].clone(), g["r"].clone()
    oracle.fused_add_rms_norm_out(x, r, g["w"], x, r, g["eps"])
    assert_bitwise_equal(r, g["res"], what=name + " residual")
    assert_ulp_close(x, g["out"], what=name)


@pytest.mark.parametrize("name", golden_names("qk_"))
def test_qk_rms_norm_rope_matches_reference(name):
    g = load_golden(name)
    q, k = g["q"].clone(), g["k"].clone()
    oracle.qk_rms_norm_rope_(q, k, g["qw"], g["kw"], g["pos"], g["cache"], g["eps"])
    assert_rope_close(q, g["q_out"], rope_bound(g["q"], g["qw"], g["pos"], g["cache"], g["q_out"]),
                      what=name + " q")
    assert_rope_close(k, g["k_out"], rope_bound(g["k"], g["kw"], g["pos"], g["cache"], g["k_out"]),
                      what=name + " k")


def test_qk_zero_input_gives_zero_output():
    for name in golden_names("qk_zero_"):
        g = load_golden(name)
        q, k = g["q"].clone(), g["k"].clone()
        oracle.qk_rms_norm_rope_(q, k, g["qw"], g["kw"], g["pos"], g["cache"], g["eps"])
        assert not q.any() and not k.any()
        assert_bitwise_equal(q, g["q_out"], what=name)


@pytest.mark.parametrize("name", golden_names("qkkv_"))
def test_qk_kv_store_matches_reference(name):
    g = load_golden(name)
    q, k, kc, vc = g["q"].clone(), g["k"].clone(), g["kc"].clone(), g["vc"].clone()
    oracle.qk_rms_norm_rope_kv_(q, k, g["v"], g["qw"], g["kw"], g["pos"], g["cache"],
                                kc, vc, g["slots"], g["eps"])
    assert_rope_close(q, g["q_out"], rope_bound(g["q"], g["qw"], g["pos"], g["cache"], g["q_out"]),
                      what=name + " q")
    assert_rope_close(k, g["k_out"], rope_bound(g["k"], g["kw"], g["pos"], g["cache"], g["k_out"]),
                      what=name + " k")
    # Written slots hold this oracle's own rotated K and the untouched V bit for
    # bit; every other slot is unchanged.
    expect_kc, expect_vc = g["kc"].clone(), g["vc"].clone()
    valid = g["slots"] >= 0
    expect_kc[g["slots"][valid].long()] = k[valid]
    expect_vc[g["slots"][valid].long()] = g["v"][valid]
    assert_bitwise_equal(kc, expect_kc, what=name + " key_cache")
    assert_bitwise_equal(vc, expect_vc, what=name + " value_cache")
    assert_bitwise_equal(vc, g["vc_out"], what=name + " value_cache vs reference")


def test_oracle_exact_match_rate_is_high():
    """Most outputs agree bit for bit; only the fp32 sum order differs."""
    total = same = 0
    for name in golden_names("fused_bf16") + golden_names("fused_fp16"):
        g = load_golden(name)
        out, _ = oracle.fused_add_rms_norm(g["x"], g["r"], g["w"], g["eps"])
        total += out.numel()
        same += int((out.view(torch.int16) == g["out"].view(torch.int16)).sum())
    assert same / total > 0.999, same / total


def test_out_of_range_positions_and_slots_are_skipped():
    torch.manual_seed(3)
    q = torch.randn(3, 2, 128, dtype=torch.bfloat16)
    k = torch.randn(3, 1, 128, dtype=torch.bfloat16)
    v = torch.randn_like(k)
    w = torch.ones(128, dtype=torch.bfloat16)
    cache = torch.randn(4, 128)
    pos = torch.tensor([0, 4, -1])           # only token 0 is in range
    slots = torch.tensor([5, 0, 1], dtype=torch.int32)   # slot 5 is past the cache
    kc = torch.zeros(4, 1, 128, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q0, k0 = q.clone(), k.clone()
    oracle.qk_rms_norm_rope_kv_(q, k, v, w, w, pos, cache, kc, vc, slots)
    assert_bitwise_equal(q[1:], q0[1:], what="skipped tokens")
    assert_bitwise_equal(k[1:], k0[1:], what="skipped tokens")
    assert not torch.equal(q[0], q0[0])
    assert not kc.any() and not vc.any()
