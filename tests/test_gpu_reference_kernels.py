"""The reference project's own CUDA kernels, compiled for sm_100a from its
sources (oracle/build_ref.py), as a second checker on the same B200.

* Residual outputs round(x + r) are bit-identical between the two builds.
* The oracle agrees with these kernels at least as closely as with the
  reference's kernels (which are built with --use_fast_math: approximate
  rsqrt and division).
* Q/K: the reference kernel rounds the normalised value once; the reference
  oracle (and these kernels) round twice. These kernels meet the propagated
  1-ulp bar everywhere; the reference kernel does not always.
"""
import pytest
import torch

from gpu_cases import expect_fused_add, expect_qk
from numerics import assert_bitwise_equal, rope_bound, rope_violations, ulp_distance
from oracle import build_ref
from sm120_rmsnorm import fused_add_rms_norm, fused_qk_rms_norm_rope_kv

pytestmark = pytest.mark.gpu
REF = build_ref.load()
needs_ref = pytest.mark.skipif(REF is None, reason="reference kernels not built")


def rand(shape, dtype, seed, mean=0.0, std=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, device="cuda", generator=g) * std + mean).to(dtype)


@needs_ref
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tokens, hidden", [(64, 1024), (256, 4096), (33, 768)])
def test_fused_add_against_the_reference_kernels(dtype, tokens, hidden):
    x, r = rand((tokens, hidden), dtype, 1), rand((tokens, hidden), dtype, 2)
    w = rand((hidden,), dtype, 3, 1.0, 0.1)
    mine_out, mine_res = fused_add_rms_norm(x, r, w)
    ref_out, ref_res = REF.fused_add_rms_norm(x, r, w, 1e-6, 0)
    assert_bitwise_equal(mine_res, ref_res, what="residual (ours vs reference kernels)")
    want, _ = expect_fused_add(x, r, w)
    mine_ulp = int(ulp_distance(mine_out.cpu(), want).max())
    ref_ulp = int(ulp_distance(ref_out.cpu(), want).max())
    assert mine_ulp <= 1
    assert mine_ulp <= ref_ulp, (mine_ulp, ref_ulp)


@needs_ref
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_qk_double_rounding_versus_the_reference_kernel(dtype):
    tokens = 256
    q = rand((tokens, 16, 128), dtype, 4)
    k = rand((tokens, 8, 128), dtype, 5)
    v = rand((tokens, 8, 128), dtype, 6)
    qw, kw = rand((128,), dtype, 7, 1.0, 0.1), rand((128,), dtype, 8, 1.0, 0.1)
    pos = torch.randperm(4096, generator=torch.Generator().manual_seed(9))[:tokens].cuda()
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
    f = torch.outer(torch.arange(4096, dtype=torch.float32, device="cuda"), inv)
    cache = torch.cat((f.cos(), f.sin()), dim=-1)
    slots = torch.arange(tokens, device="cuda", dtype=torch.int32)
    want_q, _ = expect_qk(q, k, qw, kw, pos, cache)
    bound = rope_bound(q.cpu(), qw.cpu(), pos.cpu(), cache.cpu(), want_q)

    def run(fn):
        q2, k2 = q.clone(), k.clone()
        kc = torch.zeros(tokens, 8, 128, device="cuda", dtype=dtype)
        vc = torch.zeros_like(kc)
        fn(q2, k2, v, qw, kw, pos, cache, kc, vc, slots)
        return q2, k2, kc, vc

    mq, mk, mkc, mvc = run(lambda *a: fused_qk_rms_norm_rope_kv(*a))
    rq, rk, rkc, rvc = run(lambda *a: REF.fused_qk_rms_norm_rope_kv(*a, 1e-6, 1))
    mine_bad = int(rope_violations(mq, want_q, bound).sum())
    ref_bad = int(rope_violations(rq, want_q, bound).sum())
    assert mine_bad == 0
    assert mine_bad <= ref_bad
    # both builds store their own rotated K and the unmodified V bit for bit
    assert_bitwise_equal(mkc, mk, what="key cache (ours)")
    assert_bitwise_equal(rkc, rk, what="key cache (reference)")
    assert_bitwise_equal(mvc, rvc, what="value cache")
