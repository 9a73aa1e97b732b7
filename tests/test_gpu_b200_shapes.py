"""Parity at the workload shapes the kernels are built for (B200, bf16/fp16).

Small and medium shapes are checked element for element against the oracle.
At the full prefill sizes the oracle checks a seeded sample of rows / tokens,
and size-independent properties cover every element:
  * residual_output == x + residual, bit for bit (PyTorch's own rounded add);
  * every written KV slot equals the kernel's own rotated K / input V, bit for
    bit, and every other slot is unchanged;
  * a second run on the same inputs reproduces the outputs bit for bit.
Tolerances are the ones stated in numerics.py.
"""
import pytest
import torch

from gpu_cases import (assert_bitwise_equal, check_norm, check_rope, expect_fused_add,
                       expect_qk, expect_rms_norm)
from sm120_rmsnorm import (fused_add_rms_norm_inplace, fused_add_rms_norm_out,
                           fused_qk_rms_norm_rope, fused_qk_rms_norm_rope_kv, rms_norm)

pytestmark = pytest.mark.gpu


def gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def normal(shape, dtype, g, mean=0.0, std=1.0):
    return (torch.randn(shape, device="cuda", generator=g) * std + mean).to(dtype)


def rope_cache(positions: int, theta: float = 1e6) -> torch.Tensor:
    inv_freq = 1.0 / (theta ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
    freqs = torch.outer(torch.arange(positions, dtype=torch.float32, device="cuda"), inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


# ---- RMSNorm on the CPU-runnable workload, and wide rows ------------------------

@pytest.mark.parametrize("tokens", [1, 4, 16, 64, 256])
@pytest.mark.parametrize("version", [1, 2])
def test_rms_norm_fp32_workload(tokens, version):
    g = gen(1000 + tokens)
    x = normal((tokens, 1024), torch.float32, g)
    w = normal((1024,), torch.float32, g, 1.0, 0.1)
    check_norm(rms_norm(x, w, version=version).cpu(), expect_rms_norm(x, w))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hidden", [768, 4096, 8192, 12288])
def test_rms_norm_wide(dtype, hidden):
    g = gen(hidden)
    x = normal((33, hidden), dtype, g)
    w = normal((hidden,), dtype, g, 1.0, 0.1)
    check_norm(rms_norm(x, w).cpu(), expect_rms_norm(x, w))


# ---- residual add + RMSNorm sweep: tokens x hidden x dtype ----------------------

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hidden", [768, 1024, 2048, 4096])
@pytest.mark.parametrize("tokens", [1, 4, 16, 64, 256, 1024])
@pytest.mark.parametrize("version", [0, 2])
def test_fused_add_sweep_in_place(dtype, hidden, tokens, version):
    g = gen(tokens * 7 + hidden)
    x = normal((tokens, hidden), dtype, g)
    r = normal((tokens, hidden), dtype, g)
    w = normal((hidden,), dtype, g, 1.0, 0.1)
    expected, expected_res = expect_fused_add(x, r, w)
    fused_add_rms_norm_inplace(x, r, w, version=version)
    assert_bitwise_equal(r, expected_res, what="residual")
    check_norm(x.cpu(), expected, what="output")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("hidden", [2048, 2560, 3072, 4096])
@pytest.mark.parametrize("tokens", [500, 600, 700, 900, 1200])
def test_rows_around_the_resident_grid(dtype, hidden, tokens):
    """Mid-size calls on either side of the point where the two-pack grid with
    the weight in registers stops holding every row at once (above it the
    weight is read from L1 at more blocks per SM)."""
    g = gen(tokens * 13 + hidden)
    x = normal((tokens, hidden), dtype, g)
    r = normal((tokens, hidden), dtype, g)
    w = normal((hidden,), dtype, g, 1.0, 0.1)
    check_norm(rms_norm(x, w).cpu(), expect_rms_norm(x, w), what="rms_norm")
    expected, expected_res = expect_fused_add(x, r, w)
    fused_add_rms_norm_inplace(x, r, w)
    assert_bitwise_equal(r, expected_res, what="residual")
    check_norm(x.cpu(), expected, what="output")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tokens", [1, 256, 1024])
@pytest.mark.parametrize("version", [3, 4])
def test_fused_add_h1024_versions(dtype, tokens, version):
    g = gen(tokens + version)
    x = normal((tokens, 1024), dtype, g)
    r = normal((tokens, 1024), dtype, g)
    w = normal((1024,), dtype, g, 1.0, 0.1)
    expected, expected_res = expect_fused_add(x, r, w)
    fused_add_rms_norm_inplace(x, r, w, version=version)
    assert_bitwise_equal(r, expected_res, what="residual")
    check_norm(x.cpu(), expected, what="output")


def test_fused_add_prefill_65536x8192():
    """Prefill-scale in-place residual add + RMSNorm, bf16 [65536, 8192]."""
    g = gen(65536)
    tokens, hidden = 65536, 8192
    x = normal((tokens, hidden), torch.bfloat16, g)
    r = normal((tokens, hidden), torch.bfloat16, g)
    w = normal((hidden,), torch.bfloat16, g, 1.0, 0.1)
    rows = torch.randperm(tokens, generator=torch.Generator().manual_seed(5))[:256].cuda()
    sample_x, sample_r = x[rows].clone(), r[rows].clone()
    x0, r0 = x.clone(), r.clone()
    summed = x + r  # PyTorch's bf16 add: fp32 sum rounded to nearest even
    fused_add_rms_norm_inplace(x, r, w)
    assert_bitwise_equal(r, summed, what="residual (all rows)")
    expected, _ = expect_fused_add(sample_x, sample_r, w)
    check_norm(x[rows].cpu(), expected, what="output (sampled rows)")
    # determinism: the same inputs give the same bits
    out, res = torch.empty_like(x0), torch.empty_like(r0)
    fused_add_rms_norm_out(x0, r0, w, out, res)
    assert torch.equal(out.view(torch.int16), x.view(torch.int16))
    assert torch.equal(res.view(torch.int16), r.view(torch.int16))


# ---- Q/K Norm + RoPE (+ paged KV) ----------------------------------------------

def _qk_inputs(tokens, hq, hk, dtype, seed):
    g = gen(seed)
    q = normal((tokens, hq, 128), dtype, g)
    k = normal((tokens, hk, 128), dtype, g)
    v = normal((tokens, hk, 128), dtype, g)
    qw = normal((128,), dtype, g, 1.0, 0.1)
    kw = normal((128,), dtype, g, 1.0, 0.1)
    return q, k, v, qw, kw


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("version", [1, 4])
def test_qk_kv_decode_batch1(dtype, version):
    """Qwen3 batch-1 decode: q[1,16,128], k,v[1,8,128], cache [2048,16,8,128]."""
    q, k, v, qw, kw = _qk_inputs(1, 16, 8, dtype, 4242)
    g = torch.Generator().manual_seed(4242)
    pos = torch.randint(0, 32768, (1,), generator=g).cuda()
    slots = torch.randint(0, 2048 * 16, (1,), generator=g).to(torch.int32).cuda()
    cache = rope_cache(32768)
    kc = torch.zeros((2048, 16, 8, 128), device="cuda", dtype=dtype)
    vc = torch.zeros_like(kc)
    q0, k0 = q.clone(), k.clone()
    eq, ek = expect_qk(q, k, qw, kw, pos, cache)
    fused_qk_rms_norm_rope_kv(q, k, v, qw, kw, pos, cache, kc, vc, slots, version=version)
    check_rope(q.cpu(), eq, q0, qw, pos, cache, what="query")
    check_rope(k.cpu(), ek, k0, kw, pos, cache, what="key")
    flat_k, flat_v = kc.view(-1, 8, 128), vc.view(-1, 8, 128)
    s = int(slots[0])
    assert_bitwise_equal(flat_k[s], k[0], what="key slot")
    assert_bitwise_equal(flat_v[s], v[0], what="value slot")
    flat_k[s].zero_()
    flat_v[s].zero_()
    assert not kc.any() and not vc.any(), "a slot other than slot_mapping[0] was written"


@pytest.mark.parametrize("batch", [64, 256, 1024])
def test_qk_kv_wide_decode(batch):
    """Qwen3-8B-shaped decode: q[B,32,128], k,v[B,8,128], unique slots in 65536x16."""
    dtype = torch.bfloat16
    q, k, v, qw, kw = _qk_inputs(batch, 32, 8, dtype, batch)
    g = torch.Generator().manual_seed(batch)
    pos = torch.randperm(32768, generator=g)[:batch].cuda()
    slots = torch.randperm(65536 * 16, generator=g)[:batch].to(torch.int32).cuda()
    cache = rope_cache(32768)
    kc = torch.empty((65536, 16, 8, 128), device="cuda", dtype=dtype).fill_(3.0)
    vc = torch.empty_like(kc).fill_(-3.0)
    q0, k0 = q.clone(), k.clone()
    eq, ek = expect_qk(q, k, qw, kw, pos, cache)
    fused_qk_rms_norm_rope_kv(q, k, v, qw, kw, pos, cache, kc, vc, slots)
    check_rope(q.cpu(), eq, q0, qw, pos, cache, what="query")
    check_rope(k.cpu(), ek, k0, kw, pos, cache, what="key")
    flat_k, flat_v = kc.view(-1, 8, 128), vc.view(-1, 8, 128)
    idx = slots.long()
    assert_bitwise_equal(flat_k[idx], k, what="key slots")
    assert_bitwise_equal(flat_v[idx], v, what="value slots")
    flat_k[idx] = 3.0
    flat_v[idx] = -3.0
    assert bool((kc == 3.0).all()) and bool((vc == -3.0).all()), "an unmapped slot was written"


def test_qk_kv_prefill_32768_tokens():
    """Prefill: 32768 tokens x (64 q, 8 kv) heads, positions 0..32767, contiguous slots."""
    dtype, tokens = torch.bfloat16, 32768
    q, k, v, qw, kw = _qk_inputs(tokens, 64, 8, dtype, 32768)
    pos = torch.arange(tokens, device="cuda")
    slots = torch.arange(tokens, device="cuda", dtype=torch.int32)
    cache = rope_cache(32768)
    kc = torch.zeros((2048, 16, 8, 128), device="cuda", dtype=dtype)
    vc = torch.zeros_like(kc)
    sample = torch.randperm(tokens, generator=torch.Generator().manual_seed(9))[:512].cuda()
    sq, sk, spos = q[sample].clone(), k[sample].clone(), pos[sample].clone()
    fused_qk_rms_norm_rope_kv(q, k, v, qw, kw, pos, cache, kc, vc, slots)
    eq, ek = expect_qk(sq, sk, qw, kw, spos, cache)
    check_rope(q[sample].cpu(), eq, sq, qw, spos, cache, what="query (sampled tokens)")
    check_rope(k[sample].cpu(), ek, sk, kw, spos, cache, what="key (sampled tokens)")
    assert_bitwise_equal(kc.view(tokens, 8, 128), k, what="key cache (all slots)")
    assert_bitwise_equal(vc.view(tokens, 8, 128), v, what="value cache (all slots)")


def test_qk_prefill_no_kv_matches_kv_variant():
    """The QK-only operator and the QK-KV operator produce identical Q/K bits."""
    q, k, v, qw, kw = _qk_inputs(4096, 64, 8, torch.bfloat16, 77)
    pos = torch.arange(4096, device="cuda")
    cache = rope_cache(4096)
    q2, k2 = q.clone(), k.clone()
    kc = torch.zeros((4096, 8, 128), device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    fused_qk_rms_norm_rope(q, k, qw, kw, pos, cache)
    fused_qk_rms_norm_rope_kv(q2, k2, v, qw, kw, pos, cache, kc, vc,
                              torch.arange(4096, device="cuda", dtype=torch.int32))
    assert torch.equal(q.view(torch.int16), q2.view(torch.int16))
    assert torch.equal(k.view(torch.int16), k2.view(torch.int16))


def test_qk_more_tokens_than_a_grid_dimension():
    """70000 tokens: beyond the 65535 grid.y cap the reference launch has."""
    q, k, v, qw, kw = _qk_inputs(70000, 1, 1, torch.bfloat16, 70000)
    pos = torch.arange(70000, device="cuda") % 1024
    cache = rope_cache(1024)
    q0, k0 = q.clone(), k.clone()
    eq, ek = expect_qk(q, k, qw, kw, pos, cache)
    fused_qk_rms_norm_rope(q, k, qw, kw, pos, cache)
    check_rope(q.cpu(), eq, q0, qw, pos, cache, what="query")
    check_rope(k.cpu(), ek, k0, kw, pos, cache, what="key")


# ---- rows staged in shared memory (16-128 MiB calls of 4-16 KiB rows) ------------

@pytest.mark.parametrize("rows,hidden,dtype", [
    (2048, 4096, torch.bfloat16), (2048, 4096, torch.float16), (4096, 2048, torch.bfloat16),
    (1024, 8192, torch.float16), (1024, 4096, torch.float32), (8192, 8192, torch.bfloat16)])
def test_staged_rows_match_the_oracle_and_version_2(rows, hidden, dtype):
    """The staged kernel (auto dispatch at these sizes) against the oracle on a
    sample of rows and, bit for bit on every row, against version 2 (the
    register kernel with the same threads and packs per thread)."""
    g = gen(rows + hidden)
    x = normal((rows, hidden), dtype, g)
    r = normal((rows, hidden), dtype, g)
    w = normal((hidden,), dtype, g, 1.0, 0.1)
    sample = torch.randperm(rows, generator=torch.Generator().manual_seed(rows))[:256].cuda()
    expected, expected_res = expect_fused_add(x[sample], r[sample], w)
    x2, r2 = x.clone(), r.clone()
    fused_add_rms_norm_inplace(x, r, w)
    fused_add_rms_norm_inplace(x2, r2, w, version=2)
    assert_bitwise_equal(r[sample], expected_res, what="residual (sampled rows)")
    check_norm(x[sample].cpu(), expected, what="output (sampled rows)")
    assert_bitwise_equal(r, r2, what="residual vs version 2")
    assert_bitwise_equal(x, x2, what="output vs version 2")
    # plain RMSNorm at the same size: oracle on the sample; where auto dispatch
    # stages it too (8-16 KiB rows, 16-32 MiB calls), version 1 bit for bit
    y = rms_norm(r, w)
    row_bytes = hidden * r.element_size()
    if row_bytes >= 8192 and rows * row_bytes < (32 << 20):
        assert_bitwise_equal(y, rms_norm(r, w, version=1), what="rms_norm vs version 1")
    check_norm(y[sample].cpu(), expect_rms_norm(r[sample], w), what="rms_norm (sampled rows)")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_staged_rows_out_of_place(dtype):
    """The staged kernel writing separate output / residual-output buffers
    (fused_add_rms_norm_out, fused_add_rms_norm) gives the in-place bits and
    leaves its inputs untouched."""
    g = gen(4096 + 2048)
    x = normal((2048, 4096), dtype, g)
    r = normal((2048, 4096), dtype, g)
    w = normal((4096,), dtype, g, 1.0, 0.1)
    x0, r0 = x.clone(), r.clone()
    out, res = torch.empty_like(x), torch.empty_like(x)
    fused_add_rms_norm_out(x, r, w, out, res)
    assert_bitwise_equal(x, x0, what="input untouched")
    assert_bitwise_equal(r, r0, what="residual untouched")
    fused_add_rms_norm_inplace(x, r, w)
    assert_bitwise_equal(out, x, what="output vs in place")
    assert_bitwise_equal(res, r, what="residual output vs in place")
