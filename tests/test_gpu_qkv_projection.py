"""The QKV projection on the tensor cores with the Q/K norm + RoPE + KV store
in its epilogue (csrc/qkv_gemm.cu).

Bars:
  * plain GEMM (fuse_norm=False): on inputs whose products and partial sums
    are exact in fp32 (multiples of 1/4 and 1/8 with small numerators), every
    summation order gives the same fp32 sum, so the bf16 output must equal
    PyTorch's GEMM bit for bit; on random inputs it must lie within the
    fp32 summation bound of the exact product: |out - round(exact)| <=
    ulp_bf16 + K * 2^-24 * sum |a_k w_k| (cancellation makes a pure ulp bar
    meaningless near zero).
  * fused epilogue: bit-identical to this kernel's plain GEMM followed by the
    stand-alone Q/K kernel (fused_qk_rms_norm_rope_kv on the [T, H, 128] view,
    i.e. the reference operator) -- every head, the KV caches, and the skips
    (out-of-range positions, padding slots).
"""
import pytest
import torch

import sm120_rmsnorm as ops
from numerics import assert_bitwise_equal, ulp_at
from sm120_rmsnorm import capi, extensions

pytestmark = pytest.mark.gpu
DEV = "cuda"


def operands(tokens, hidden, hq, hk, seed, exact):
    g = torch.Generator(device=DEV).manual_seed(seed)
    n = (hq + 2 * hk) * 128
    if exact:
        a = torch.randint(-3, 4, (tokens, hidden), device=DEV, generator=g).float() / 4
        w = torch.randint(-3, 4, (n, hidden), device=DEV, generator=g).float() / 8
    else:
        a = torch.randn(tokens, hidden, device=DEV, generator=g)
        w = torch.randn(n, hidden, device=DEV, generator=g) / hidden ** 0.5
    return a.bfloat16(), w.bfloat16()


def rope_table(positions=4096):
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device=DEV) / 128))
    f = torch.outer(torch.arange(positions, dtype=torch.float32, device=DEV), inv)
    return torch.cat((f.cos(), f.sin()), dim=-1)


# Launch forms (csrc/qkv_gemm.cu): up to four tokens with hidden a multiple
# of 512 stream the weights on the CUDA cores (the 1-, 2-, 3- and 4-token
# cases here); otherwise a wave model picks, from the plain GEMM's costs,
# 4-way split K over one-head tiles (5, 7, 8, 37, 64, 128 tokens, and 300
# tokens with 8 heads) or 2-way split K (257 tokens with 48 heads), else an
# unsplit form by the call's own costs: two-head tiles (513, 700, 1000
# tokens, fused 1300 x 512), one 256 x 256 tile per CTA pair (plain 1300
# tokens -- the second CTA of the last pair has no token rows -- and plain
# 2048 x 1024), or the
# persistent CTA pairs with two accumulators (plain 2048 x 2048 and 2048 x
# 4096; fused 2048 x 1024: three rounds of 74 clusters; fused 512 x 4096:
# fewer tiles than clusters; fused 4000 x 512: six rounds, so each
# accumulator cycles three times). Fused and plain calls of one shape thus
# sum K in the same order, which the bit-for-bit comparison below needs.
# Hidden 64 (K not a multiple of 256) cannot split and runs on one-head
# tiles.
@pytest.mark.parametrize("tokens, hidden, hq, hk", [
    (1, 64, 2, 0), (128, 256, 2, 1), (300, 1024, 4, 2), (257, 4096, 32, 8), (1000, 2048, 16, 8),
    (1300, 512, 32, 8), (2048, 1024, 32, 8), (1, 512, 2, 1), (5, 1024, 4, 2), (8, 4096, 32, 8),
    (2, 8192, 4, 2), (4, 8192, 8, 4), (2048, 2048, 32, 8)])
def test_plain_gemm_is_exact_on_exact_inputs(tokens, hidden, hq, hk):
    a, w = operands(tokens, hidden, hq, hk, tokens, exact=True)
    out = torch.zeros(tokens, w.shape[0], device=DEV, dtype=torch.bfloat16)
    extensions.qkv_proj_norm_rope_cache_(a, w, out, hq, hk, fuse_norm=False)
    assert_bitwise_equal(out, a @ w.t(), what="GEMM")


@pytest.mark.parametrize("tokens, hidden", [(1, 4096), (2, 4096), (7, 2048), (64, 4096),
                                           (513, 1024), (1300, 1024), (2048, 4096)])
def test_plain_gemm_random_inputs_within_one_ulp(tokens, hidden):
    a, w = operands(tokens, hidden, 32, 8, 5, exact=False)
    out = torch.empty(tokens, w.shape[0], device=DEV, dtype=torch.bfloat16)
    extensions.qkv_proj_norm_rope_cache_(a, w, out, 32, 8, fuse_norm=False)
    exact = a.double() @ w.double().t()
    magnitude = a.double().abs() @ w.double().abs().t()
    want = exact.bfloat16()
    ulp = ulp_at(torch.maximum(exact.abs(), want.double().abs()).cpu(), torch.bfloat16)
    bound = ulp + hidden * 2.0 ** -24 * magnitude.cpu()
    err = (out.double() - want.double()).abs().cpu()
    assert bool((err <= bound).all()), float((err - bound).max())
    assert float((out != want).float().mean()) < 0.01  # nearly all bit-identical


@pytest.mark.parametrize("tokens, hidden, hq, hk", [
    (1, 256, 16, 8), (37, 1024, 8, 4), (128, 4096, 32, 8), (700, 2048, 16, 8),
    (1300, 512, 32, 8), (2048, 1024, 32, 8), (1, 4096, 32, 8), (3, 1024, 8, 4), (8, 512, 16, 8),
    (4, 8192, 8, 4), (257, 4096, 32, 8), (512, 4096, 32, 8), (4000, 512, 32, 8)])
@pytest.mark.parametrize("with_cache", [True, False])
def test_fused_epilogue_equals_gemm_then_qk_kernel(tokens, hidden, hq, hk, with_cache):
    a, w = operands(tokens, hidden, hq, hk, 7 + tokens, exact=False)
    g = torch.Generator(device=DEV).manual_seed(tokens)
    qw = (1 + 0.1 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    kw = (1 + 0.1 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    table = rope_table()
    pos = torch.randint(0, 4096, (tokens,), device=DEV, generator=g)
    if tokens > 1:
        pos[0] = -1              # out of range: the token stays the plain GEMM output
    if tokens > 2:
        pos[1] = 4096
    slots_total = (tokens + 16) * 2
    slots = torch.randperm(slots_total, device=DEV, generator=g)[:tokens].to(torch.int32)
    if tokens > 3:
        slots[3] = -1            # padding token: no store
    n = w.shape[0]

    fused = torch.zeros(tokens, n, device=DEV, dtype=torch.bfloat16)
    kc = torch.zeros(slots_total, hk, 128, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    caches = (kc, vc, slots) if with_cache else (None, None, None)
    extensions.qkv_proj_norm_rope_cache_(a, w, fused, hq, hk, qw, kw, pos, table, *caches)

    plain = torch.zeros(tokens, n, device=DEV, dtype=torch.bfloat16)
    extensions.qkv_proj_norm_rope_cache_(a, w, plain, hq, hk, fuse_norm=False)
    heads = plain.view(tokens, hq + 2 * hk, 128)
    q, k, v = (heads[:, :hq].contiguous(), heads[:, hq:hq + hk].contiguous(),
               heads[:, hq + hk:].contiguous())
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    if with_cache:
        ops.fused_qk_rms_norm_rope_kv(q, k, v, qw, kw, pos, table, kc2, vc2, slots)
    else:
        ops.fused_qk_rms_norm_rope(q, k, qw, kw, pos, table)
    want = torch.cat((q, k, v), dim=1).view(tokens, n)
    assert_bitwise_equal(fused, want, what="qkv")
    assert_bitwise_equal(kc, kc2, what="key cache")
    assert_bitwise_equal(vc, vc2, what="value cache")
    assert capi.device_faults() == 0


def test_back_to_back_calls_and_graph_capture():
    """Two launches in a row (the second overlapping the first's tail under
    programmatic launch) and a captured graph give the same result."""
    a, w = operands(256, 2048, 16, 8, 3, exact=False)
    g = torch.Generator(device=DEV).manual_seed(3)
    qw = (1 + 0.1 * torch.randn(128, device=DEV, generator=g)).bfloat16()
    pos = torch.randint(0, 4096, (256,), device=DEV, generator=g)
    table = rope_table()
    outs = [torch.zeros(256, w.shape[0], device=DEV, dtype=torch.bfloat16) for _ in range(3)]
    for out in outs[:2]:
        extensions.qkv_proj_norm_rope_cache_(a, w, out, 16, 8, qw, qw, pos, table)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        extensions.qkv_proj_norm_rope_cache_(a, w, outs[2], 16, 8, qw, qw, pos, table)
    graph.replay()
    torch.cuda.synchronize()
    assert_bitwise_equal(outs[1], outs[0], what="second launch")
    assert_bitwise_equal(outs[2], outs[0], what="graph replay")


def test_argument_checks():
    a = torch.zeros(4, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(384, 64, device=DEV, dtype=torch.bfloat16)
    out = torch.zeros(4, 384, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="even number of heads"):
        extensions.qkv_proj_norm_rope_cache_(a, w, out, 1, 1, fuse_norm=False)
    a2 = torch.zeros(4, 96, device=DEV, dtype=torch.bfloat16)
    w2 = torch.zeros(512, 96, device=DEV, dtype=torch.bfloat16)
    out2 = torch.zeros(4, 512, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="multiple of 64"):
        extensions.qkv_proj_norm_rope_cache_(a2, w2, out2, 2, 1, fuse_norm=False)
    with pytest.raises(RuntimeError, match="the fused norm needs"):
        extensions.qkv_proj_norm_rope_cache_(a2, w2, out2, 2, 1)
