"""GPU parity of the engine-side extensions (csrc/head_cache.cu,
csrc/norm_quant.cu) against the extension oracle (oracle/extensions.py).

Bars:
  * exact-sum inputs (multiples of 1/16 small enough that every square and
    every partial sum of squares is exact in fp32, so no summation order can
    change inv_rms): Q/K outputs, caches, fp8 codes, token scales and
    residuals all bit-identical to the oracle;
  * random inputs: Q/K within the propagated RoPE bound (tests/numerics.py),
    caches bit-identical to the kernel's own rotated K / the input V (fp8:
    to their conversion by the oracle), fp8 codes at most one e4m3 step from
    the oracle's, dynamic scales within one ulp of the activation dtype
    (relative) of the oracle's;
  * at head_dim = rotary_dim = 128, NEOX, same-dtype NHD caches and dense
    inputs: bit-identical to ops.fused_qk_rms_norm_rope_kv.
"""
import pytest
import torch

from numerics import assert_bitwise_equal, assert_rope_close, rope_bound
from oracle import extensions as ex
from sm120_rmsnorm import extensions, fused_qk_rms_norm_rope_kv

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def gen(seed):
    return torch.Generator().manual_seed(seed)


def exact_values(shape, dtype, g, limit=32):
    """k / 16 for integer k in [-limit, limit]."""
    return (torch.randint(-limit, limit + 1, shape, generator=g).float() / 16).to(dtype)


def weights(n, dtype, g):
    return (1 + 0.1 * torch.randn(n, generator=g)).to(dtype)


def cos_sin(positions, rotary, base=1e6):
    inv = 1.0 / (base ** (torch.arange(0, rotary, 2, dtype=torch.float32) / rotary))
    f = torch.outer(torch.arange(positions, dtype=torch.float32), inv)
    return torch.cat((f.cos(), f.sin()), dim=-1)


def e4m3_step_distance(a, b):
    def ordered(t):
        c = t.cpu().contiguous().view(torch.uint8).to(torch.int16)
        return torch.where(c >= 128, -(c & 0x7F), c)
    return (ordered(a) - ordered(b)).abs()


class QkCase:
    """Inputs of one qk_norm_rope_cache call on CPU; `run` applies the GPU
    operator to device copies (optionally as views into one QKV buffer)."""

    def __init__(self, dtype, head_dim, rotary, tokens=33, hq=4, hk=2, exact=True, seed=0,
                 layout="NHD", cache="same", blocks=8, block_size=16, neox=True):
        g = gen(seed)
        make = (lambda s: exact_values(s, dtype, g)) if exact else (
            lambda s: torch.randn(s, generator=g).to(dtype))
        self.dtype, self.layout, self.neox = dtype, layout, neox
        self.q, self.k, self.v = make((tokens, hq, head_dim)), make((tokens, hk, head_dim)), \
            make((tokens, hk, head_dim))
        self.qw, self.kw = weights(head_dim, dtype, g), weights(head_dim, dtype, g)
        self.table = cos_sin(4096, rotary)
        self.pos = torch.randint(0, 4096, (tokens,), generator=g)
        capacity = blocks * block_size
        self.slots = torch.randperm(capacity, generator=g)[:tokens].to(torch.int32)
        shape = (blocks, block_size, hk, head_dim) if layout == "NHD" else \
            (blocks, hk, block_size, head_dim)
        cache_dtype = {"same": dtype, "fp8": torch.float8_e4m3fn, "u8": torch.uint8}[cache]
        self.kc = torch.zeros(shape, dtype=cache_dtype)
        self.vc = torch.zeros(shape, dtype=cache_dtype)
        self.k_scale = torch.tensor([0.75]) if cache != "same" else None
        self.v_scale = torch.tensor([0.0625]) if cache != "same" else None

    def expected(self):
        return ex.qk_norm_rope_cache(self.q, self.k, self.v, self.qw, self.kw, self.pos,
                                     self.table, self.kc, self.vc, self.slots, self.k_scale,
                                     self.v_scale, self.neox, self.layout)

    def run(self, strided=False):
        if strided:
            t, hq, d = self.q.shape
            hk = self.k.shape[1]
            qkv = torch.cat((self.q.reshape(t, -1), self.k.reshape(t, -1),
                             self.v.reshape(t, -1)), dim=1).to(DEV)
            q = qkv[:, :hq * d].view(t, hq, d)
            k = qkv[:, hq * d:(hq + hk) * d].view(t, hk, d)
            v = qkv[:, (hq + hk) * d:].view(t, hk, d)
            assert not q.is_contiguous() or t == 1
        else:
            q, k, v = self.q.to(DEV), self.k.to(DEV), self.v.to(DEV)
        kc, vc = self.kc.to(DEV), self.vc.to(DEV)
        scales = [s.to(DEV) if s is not None else None for s in (self.k_scale, self.v_scale)]
        extensions.qk_norm_rope_cache_(q, k, v, self.qw.to(DEV), self.kw.to(DEV),
                                       self.pos.to(DEV), self.table.to(DEV), kc, vc,
                                       self.slots.to(DEV), *scales, is_neox=self.neox,
                                       kv_cache_layout=self.layout)
        return q.cpu(), k.cpu(), kc.cpu(), vc.cpu()


def _rotaries(d):
    return sorted({d, d // 2, 16})


# ---- bit-identity with the reference-API kernel ------------------------------------------
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tokens", [1, 37, 1000])
def test_generalised_kernel_is_the_reference_api_kernel_at_head_dim_128(dtype, tokens):
    c = QkCase(dtype, 128, 128, tokens=tokens, hq=16, hk=8, exact=False, seed=tokens,
               blocks=(tokens + 15) // 16 + 1)
    gq, gk, gkc, gvc = c.run()
    q, k, v = c.q.to(DEV), c.k.to(DEV), c.v.to(DEV)
    kc, vc = c.kc.to(DEV), c.vc.to(DEV)
    fused_qk_rms_norm_rope_kv(q, k, v, c.qw.to(DEV), c.kw.to(DEV), c.pos.to(DEV),
                              c.table.to(DEV), kc, vc, c.slots.to(DEV))
    for got, want, what in ((gq, q, "query"), (gk, k, "key"), (gkc, kc, "key cache"),
                            (gvc, vc, "value cache")):
        assert_bitwise_equal(got, want, what=what)


# ---- exact-sum inputs: bit-identical to the oracle -----------------------------------------
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("head_dim, rotary", [(d, r) for d in (64, 128, 256) for r in _rotaries(d)])
def test_head_sizes_and_rotary_widths_exact(dtype, neox, head_dim, rotary):
    c = QkCase(dtype, head_dim, rotary, neox=neox, seed=head_dim + rotary)
    want = c.expected()
    got = c.run()
    for g_, w_, what in zip(got, want, ("query", "key", "key cache", "value cache")):
        assert_bitwise_equal(g_, w_, what=what)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout", ["NHD", "HND"])
@pytest.mark.parametrize("cache", ["same", "fp8", "u8"])
@pytest.mark.parametrize("strided", [False, True])
def test_cache_layouts_dtypes_and_strided_views_exact(dtype, layout, cache, strided):
    c = QkCase(dtype, 128, 64, layout=layout, cache=cache, seed=7, hq=8, hk=2)
    want = c.expected()
    got = c.run(strided=strided)
    for g_, w_, what in zip(got, want, ("query", "key", "key cache", "value cache")):
        if g_.dtype in (torch.float8_e4m3fn, torch.uint8):
            g_, w_ = g_.view(torch.uint8), w_.view(torch.uint8)
            assert torch.equal(g_, w_), what
        else:
            assert_bitwise_equal(g_, w_, what=what)


@pytest.mark.parametrize("layout", ["NHD", "HND"])
@pytest.mark.parametrize("cache", ["same", "fp8"])
def test_combined_kv_pages(layout, cache):
    """FlashInfer's paged layout keeps K and V of a page together:
    [pages, 2, page_size, Hk, D] ("NHD") or [pages, 2, Hk, page_size, D]
    ("HND"); key_cache = kv[:, 0] and value_cache = kv[:, 1] are strided views
    (block stride 2 x page), written in place and nothing else."""
    c = QkCase(torch.bfloat16, 128, 128, tokens=45, layout=layout, cache=cache, seed=11,
               hq=8, hk=2, blocks=6, block_size=16)
    want = c.expected()
    pages = torch.zeros((c.kc.shape[0], 2) + tuple(c.kc.shape[1:]), dtype=c.kc.dtype, device=DEV)
    kc, vc = pages[:, 0], pages[:, 1]
    assert not kc.is_contiguous()
    scales = [s.to(DEV) if s is not None else None for s in (c.k_scale, c.v_scale)]
    q, k, v = c.q.to(DEV), c.k.to(DEV), c.v.to(DEV)
    extensions.qk_norm_rope_cache_(q, k, v, c.qw.to(DEV), c.kw.to(DEV), c.pos.to(DEV),
                                   c.table.to(DEV), kc, vc, c.slots.to(DEV), *scales,
                                   kv_cache_layout=layout)
    got = (q.cpu(), k.cpu(), kc.cpu(), vc.cpu())
    for g_, w_, what in zip(got, want, ("query", "key", "key cache", "value cache")):
        if g_.dtype in (torch.float8_e4m3fn, torch.uint8):
            assert torch.equal(g_.contiguous().view(torch.uint8), w_.view(torch.uint8)), what
        else:
            assert_bitwise_equal(g_.contiguous(), w_, what=what)


@pytest.mark.parametrize("block_size", [1, 5, 16, 32])
@pytest.mark.parametrize("layout", ["NHD", "HND"])
def test_block_sizes(block_size, layout):
    c = QkCase(torch.bfloat16, 64, 64, tokens=40, layout=layout, block_size=block_size,
               blocks=(80 + block_size - 1) // block_size, seed=block_size)
    want = c.expected()
    got = c.run()
    for g_, w_, what in zip(got, want, ("query", "key", "key cache", "value cache")):
        assert_bitwise_equal(g_, w_, what=what)


# ---- random inputs: propagated bound, exact caches ---------------------------------------
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("head_dim, rotary, neox", [(64, 64, True), (256, 128, False),
                                                    (128, 32, True), (256, 256, True)])
def test_random_inputs_within_the_rope_bound(dtype, head_dim, rotary, neox):
    c = QkCase(dtype, head_dim, rotary, tokens=300, hq=8, hk=4, exact=False, seed=3,
               neox=neox, cache="u8", blocks=32)
    want_q, want_k, _, _ = c.expected()
    gq, gk, gkc, gvc = c.run()
    for got, want, x, w, what in ((gq, want_q, c.q, c.qw, "query"), (gk, want_k, c.k, c.kw, "key")):
        bound = rope_bound(x, w, c.pos, c.table, want, interleaved=not neox)
        assert_rope_close(got, want, bound, what=what)
    # the caches hold the kernel's own rotated K and the input V, quantised
    expect_kc = torch.zeros_like(c.kc)
    expect_vc = torch.zeros_like(c.vc)
    slots = c.slots.long()
    block, offset = slots // c.kc.size(1), slots % c.kc.size(1)
    expect_kc[block, offset] = ex.fp8_e4m3(gk.float() / 0.75).view(torch.uint8)
    expect_vc[block, offset] = ex.fp8_e4m3(c.v.float() / 0.0625).view(torch.uint8)
    assert torch.equal(gkc, expect_kc)
    assert torch.equal(gvc, expect_vc)


# ---- edges ------------------------------------------------------------------------------
@pytest.mark.parametrize("cache,rotary", [("same", 128), ("fp8", 128), ("fp8", 64)])
def test_out_of_range_positions_and_slots_are_skipped(cache, rotary):
    """Whole-head NEOX rotary (the compile-time form, which reads V before the
    slot is known) and partial rotary (the general form), same-type and fp8
    caches: out-of-range positions leave the token untouched, out-of-range
    slots store nothing."""
    c = QkCase(torch.bfloat16, 128, rotary, tokens=6, exact=True, seed=4, blocks=2, cache=cache)
    c.pos = torch.tensor([-1, 4096, 5, 10_000, 0, 7])
    c.slots = torch.tensor([0, 1, -1, 2, 32, 31], dtype=torch.int32)  # 32 slots in the cache
    want = c.expected()
    got = c.run()
    for g_, w_, what in zip(got, want, ("query", "key", "key cache", "value cache")):
        assert_bitwise_equal(g_, w_, what=what)
    assert_bitwise_equal(got[0][[0, 1, 3]], c.q[[0, 1, 3]], what="untouched tokens")
    written = (got[2].float() != 0).reshape(-1, *got[2].shape[2:]).flatten(1).any(-1)
    assert written.nonzero().flatten().tolist() == [31]  # only token 5 stored (slot 31)


def test_no_cache_and_no_key_heads():
    c = QkCase(torch.float16, 256, 128, tokens=9, hk=0, seed=12)
    q = c.q.to(DEV)
    k = c.k.to(DEV)
    extensions.qk_norm_rope_cache_(q, k, None, c.qw.to(DEV), c.kw.to(DEV), c.pos.to(DEV),
                                   c.table.to(DEV))
    want_q, _, _, _ = ex.qk_norm_rope_cache(c.q, c.k, None, c.qw, c.kw, c.pos, c.table)
    assert_bitwise_equal(q, want_q, what="query")


def test_unaligned_views_take_the_element_path():
    c = QkCase(torch.bfloat16, 64, 32, tokens=17, seed=13, hq=3, hk=1)
    want = c.expected()
    buf_q = torch.zeros(c.q.numel() + 1, dtype=c.dtype, device=DEV)
    buf_k = torch.zeros(c.k.numel() + 1, dtype=c.dtype, device=DEV)
    q = buf_q[1:].view(c.q.shape).copy_(c.q)
    k = buf_k[1:].view(c.k.shape).copy_(c.k)
    kc, vc = c.kc.to(DEV), c.vc.to(DEV)
    extensions.qk_norm_rope_cache_(q, k, c.v.to(DEV), c.qw.to(DEV), c.kw.to(DEV),
                                   c.pos.to(DEV), c.table.to(DEV), kc, vc, c.slots.to(DEV))
    for g_, w_, what in zip((q, k, kc, vc), want, ("query", "key", "key cache", "value cache")):
        assert_bitwise_equal(g_, w_, what=what)


def test_graph_capture_replays_the_same_result():
    c = QkCase(torch.bfloat16, 128, 128, tokens=8, hq=16, hk=8, seed=14, cache="fp8")
    want = c.expected()
    q0, k0 = c.q.to(DEV), c.k.to(DEV)
    q, k, v = q0.clone(), k0.clone(), c.v.to(DEV)
    kc, vc = c.kc.to(DEV), c.vc.to(DEV)
    args = (c.qw.to(DEV), c.kw.to(DEV), c.pos.to(DEV), c.table.to(DEV), kc, vc,
            c.slots.to(DEV), c.k_scale.to(DEV), c.v_scale.to(DEV))
    extensions.qk_norm_rope_cache_(q, k, v, *args)  # warm up outside the capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        extensions.qk_norm_rope_cache_(q, k, v, *args)
    q.copy_(q0)
    k.copy_(k0)
    kc.zero_()
    vc.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for g_, w_, what in zip((q, k), want[:2], ("query", "key")):
        assert_bitwise_equal(g_, w_, what=what)
    assert torch.equal(kc.view(torch.uint8).cpu(), want[2].view(torch.uint8))


def test_tensor_checks():
    c = QkCase(torch.bfloat16, 128, 128, tokens=4, seed=15)
    q, k, v = c.q.to(DEV), c.k.to(DEV), c.v.to(DEV)
    args = [c.qw.to(DEV), c.kw.to(DEV), c.pos.to(DEV), c.table.to(DEV)]
    kc, vc = c.kc.to(DEV), c.vc.to(DEV)
    with pytest.raises(RuntimeError, match="kv_cache_layout"):
        extensions.qk_norm_rope_cache_(q, k, v, *args, kc, vc, c.slots.to(DEV),
                                       kv_cache_layout="NDH")
    with pytest.raises(RuntimeError, match="fp8 caches need k_scale"):
        extensions.qk_norm_rope_cache_(q, k, v, *args, kc.to(torch.uint8), vc.to(torch.uint8),
                                       c.slots.to(DEV))
    with pytest.raises(RuntimeError, match="head_dim must be 64, 128 or 256"):
        extensions.qk_norm_rope_cache_(q[..., :96].contiguous(), k[..., :96].contiguous(), None,
                                       args[0][:96], args[1][:96], args[2],
                                       cos_sin(16, 96).to(DEV))
    with pytest.raises(RuntimeError, match="heads must be adjacent"):
        extensions.qk_norm_rope_cache_(q.transpose(0, 1), k.transpose(0, 1), None, *args)


# ---- RMSNorm + fp8 quantisation ------------------------------------------------------------
QUANT_HIDDEN = [64, 768, 1024, 1001, 4096, 8192, 16384, 32768]


def run_quant(x, w, residual=None, scale=None, scale_ub=None):
    x_d, w_d = x.to(DEV), w.to(DEV)
    out = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=DEV)
    r_d = residual.to(DEV) if residual is not None else None
    if scale is not None:
        if r_d is None:
            extensions.rms_norm_static_fp8_quant(out, x_d, w_d, scale.to(DEV))
        else:
            extensions.fused_add_rms_norm_static_fp8_quant(out, x_d, r_d, w_d, scale.to(DEV))
        scales = None
    else:
        scales = torch.empty(x.numel() // x.shape[-1], dtype=torch.float32, device=DEV)
        extensions.rms_norm_dynamic_per_token_quant(
            out, x_d, w_d, scales, 1e-6, scale_ub.to(DEV) if scale_ub is not None else None, r_d)
        scales = scales.cpu()
    assert torch.equal(x_d.cpu(), x), "input must not change"
    return out.cpu(), scales, (r_d.cpu() if r_d is not None else None)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("hidden", QUANT_HIDDEN)
@pytest.mark.parametrize("add", [False, True])
@pytest.mark.parametrize("dynamic", [False, True])
def test_norm_quant_exact(dtype, hidden, add, dynamic):
    g = gen(hidden)
    rows = 37
    limit = 8 if add else 16
    x = exact_values((rows, hidden), dtype, g, limit)
    r = exact_values((rows, hidden), dtype, g, limit) if add else None
    w = weights(hidden, dtype, g)
    scale = None if dynamic else torch.tensor([0.02])
    q, scales, r_out = run_quant(x, w, r, scale)
    want_q, want_scales, want_r = ex.rms_norm_fp8_quant(x, w, residual=r, scale=scale)
    assert torch.equal(q.view(torch.uint8), want_q.view(torch.uint8))
    if dynamic:
        assert_bitwise_equal(scales, want_scales.reshape(-1), what="token scales")
    if add:
        assert_bitwise_equal(r_out, want_r, what="residual")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("add", [False, True])
@pytest.mark.parametrize("dynamic", [False, True])
def test_norm_quant_many_wide_rows_exact(dtype, add, dynamic):
    """1200 rows of 8192: more than eight rows per SM, the many-row launch (a
    256-thread block per row, four packs per thread)."""
    g = gen(8192 + add + 2 * dynamic)
    limit = 8 if add else 16
    x = exact_values((1200, 8192), dtype, g, limit)
    r = exact_values((1200, 8192), dtype, g, limit) if add else None
    w = weights(8192, dtype, g)
    scale = None if dynamic else torch.tensor([0.03])
    q, scales, r_out = run_quant(x, w, r, scale)
    want_q, want_scales, want_r = ex.rms_norm_fp8_quant(x, w, residual=r, scale=scale)
    assert torch.equal(q.view(torch.uint8), want_q.view(torch.uint8))
    if dynamic:
        assert_bitwise_equal(scales, want_scales.reshape(-1), what="token scales")
    if add:
        assert_bitwise_equal(r_out, want_r, what="residual")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,hidden", [(500, 4096), (600, 4096), (1150, 4096), (1150, 3072),
                                         (1150, 2048)])
@pytest.mark.parametrize("add", [False, True])
@pytest.mark.parametrize("dynamic", [False, True])
def test_norm_quant_mid_rows_exact(dtype, rows, hidden, add, dynamic):
    """Two-pack calls on either side of the point where the blocks holding the
    weight in registers stop covering every row at once (dynamic scales then
    read the weight from L1 at more blocks per SM)."""
    g = gen(rows + hidden + add + 2 * dynamic)
    limit = 8 if add else 16
    x = exact_values((rows, hidden), dtype, g, limit)
    r = exact_values((rows, hidden), dtype, g, limit) if add else None
    w = weights(hidden, dtype, g)
    scale = None if dynamic else torch.tensor([0.03])
    q, scales, r_out = run_quant(x, w, r, scale)
    want_q, want_scales, want_r = ex.rms_norm_fp8_quant(x, w, residual=r, scale=scale)
    assert torch.equal(q.view(torch.uint8), want_q.view(torch.uint8))
    if dynamic:
        assert_bitwise_equal(scales, want_scales.reshape(-1), what="token scales")
    if add:
        assert_bitwise_equal(r_out, want_r, what="residual")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("hidden", [1024, 4096, 32768])
@pytest.mark.parametrize("dynamic", [False, True])
def test_norm_quant_random_inputs(dtype, hidden, dynamic):
    g = gen(7 + hidden)
    x = torch.randn(64, hidden, generator=g).to(dtype)
    r = torch.randn(64, hidden, generator=g).to(dtype)
    w = weights(hidden, dtype, g)
    scale = None if dynamic else torch.tensor([0.01])
    q, scales, r_out = run_quant(x, w, r, scale)
    want_q, want_scales, want_r = ex.rms_norm_fp8_quant(x, w, residual=r, scale=scale)
    assert_bitwise_equal(r_out, want_r, what="residual")
    assert int(e4m3_step_distance(q, want_q).max()) <= 1
    if dynamic:
        ulp = {torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10, torch.float32: 2.0 ** -21}[dtype]
        rel = ((scales - want_scales.reshape(-1)).abs() / want_scales.reshape(-1)).max().item()
        assert rel <= ulp


def test_norm_quant_scale_bound_zero_rows_and_saturation():
    g = gen(21)
    x = torch.randn(4, 512, generator=g).to(torch.bfloat16)
    x[1] = 0
    x[2, 7] = 300.0  # a row dominated by one outlier
    w = weights(512, torch.bfloat16, g)
    ub = torch.tensor([0.5])
    q, scales, _ = run_quant(x, w, scale_ub=ub)
    want_q, want_scales, _ = ex.rms_norm_fp8_quant(x, w, scale_ub=ub)
    assert_bitwise_equal(scales, want_scales, what="bounded scales")
    assert scales[1].item() == ex.MIN_TOKEN_SCALE
    assert int(e4m3_step_distance(q, want_q).max()) <= 1
    q_static, _, _ = run_quant(x, w, scale=torch.tensor([1e-4]))  # everything saturates
    assert q_static.float().abs().max().item() == 448.0


def test_norm_quant_empty_and_unaligned_output():
    w = torch.ones(256, dtype=torch.bfloat16)
    empty = torch.empty(0, 256, dtype=torch.bfloat16)
    q, _, _ = run_quant(empty, w, scale=torch.tensor([1.0]))
    assert q.shape == (0, 256)
    g = gen(22)
    x = exact_values((9, 256), torch.bfloat16, g)
    buf = torch.empty(9 * 256 + 1, dtype=torch.float8_e4m3fn, device=DEV)
    out = buf[1:].view(9, 256)
    extensions.rms_norm_static_fp8_quant(out, x.to(DEV), w.to(DEV), torch.tensor([0.05], device=DEV))
    want_q, _, _ = ex.rms_norm_fp8_quant(x, w, scale=torch.tensor([0.05]))
    assert torch.equal(out.cpu().view(torch.uint8), want_q.view(torch.uint8))


# ---- RMSNorm + NVFP4 -----------------------------------------------------------------
def run_fp4(x, w, g, residual=None, tiled=True):
    rows, hidden = x.numel() // x.shape[-1], x.shape[-1]
    out = torch.zeros(rows, hidden // 2, dtype=torch.uint8, device=DEV)
    scales = torch.zeros(extensions.nvfp4_scale_bytes(rows, hidden, tiled), dtype=torch.uint8,
                         device=DEV)
    r_d = residual.to(DEV) if residual is not None else None
    x_d = x.to(DEV)
    extensions.rms_norm_nvfp4_quant(out, scales, x_d, w.to(DEV), torch.tensor([g], device=DEV),
                                    1e-6, r_d, tiled)
    assert torch.equal(x_d.cpu(), x), "input must not change"
    return out.cpu(), scales.cpu(), (r_d.cpu() if r_d is not None else None)


def e2m1_step_distance(a, b):
    def nibbles(t):
        t = t.to(torch.int16)
        codes = torch.stack((t & 0xF, t >> 4), -1)
        return torch.where(codes >= 8, -(codes & 7), codes)
    return (nibbles(a) - nibbles(b)).abs()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("hidden", [64, 1024, 4096, 8192, 16384, 32768])
@pytest.mark.parametrize("add", [False, True])
@pytest.mark.parametrize("tiled", [True, False])
def test_nvfp4_exact(dtype, hidden, add, tiled):
    g = gen(hidden + add)
    limit = 8 if add else 16
    x = exact_values((37, hidden), dtype, g, limit)
    r = exact_values((37, hidden), dtype, g, limit) if add else None
    w = weights(hidden, dtype, g)
    q, scales, r_out = run_fp4(x, w, 300.0, r, tiled)
    want_q, want_scales, want_r = ex.rms_norm_nvfp4_quant(x, w, 300.0, residual=r, tiled=tiled)
    assert torch.equal(scales, want_scales), "block scales"
    assert torch.equal(q, want_q), "e2m1 codes"
    if add:
        assert_bitwise_equal(r_out, want_r, what="residual")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("add", [False, True])
def test_nvfp4_many_wide_rows_exact(dtype, add):
    """1200 rows of 8192 (the many-row launch: a 256-thread block per row, four
    packs per thread), tiled scales over a row count that is not a multiple of
    128."""
    g = gen(1200 + add)
    limit = 8 if add else 16
    x = exact_values((1200, 8192), dtype, g, limit)
    r = exact_values((1200, 8192), dtype, g, limit) if add else None
    w = weights(8192, dtype, g)
    q, scales, r_out = run_fp4(x, w, 500.0, r, True)
    want_q, want_scales, want_r = ex.rms_norm_nvfp4_quant(x, w, 500.0, residual=r, tiled=True)
    assert torch.equal(scales, want_scales)
    assert torch.equal(q, want_q)
    if add:
        assert_bitwise_equal(r_out, want_r, what="residual")


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("hidden", [1024, 8192, 32768])
def test_nvfp4_random_inputs(dtype, hidden):
    g = gen(11 + hidden)
    x = torch.randn(64, hidden, generator=g).to(dtype)
    r = torch.randn(64, hidden, generator=g).to(dtype)
    w = weights(hidden, dtype, g)
    q, scales, r_out = run_fp4(x, w, 400.0, r, False)
    want_q, want_scales, want_r = ex.rms_norm_nvfp4_quant(x, w, 400.0, residual=r, tiled=False)
    assert_bitwise_equal(r_out, want_r, what="residual")
    scale_steps = e4m3_step_distance(scales, want_scales)
    assert int(scale_steps.max()) <= 1
    assert float((scale_steps > 0).float().mean()) < 0.01
    same_scale = (scale_steps == 0).reshape(64, hidden // 16)
    steps = e2m1_step_distance(q, want_q).reshape(64, hidden // 16, 16)
    assert int(steps[same_scale].max()) <= 1


def test_nvfp4_tensor_checks():
    x = torch.randn(4, 72, device=DEV).to(torch.bfloat16)
    w = torch.ones(72, device=DEV, dtype=torch.bfloat16)
    out = torch.zeros(4, 36, dtype=torch.uint8, device=DEV)
    scales = torch.zeros(4096, dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError, match="multiple of 16"):
        extensions.rms_norm_nvfp4_quant(out, scales, x, w, torch.ones(1, device=DEV))
    x = torch.randn(4, 64, device=DEV).to(torch.bfloat16)
    w = torch.ones(64, device=DEV, dtype=torch.bfloat16)
    out = torch.zeros(4, 32, dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError, match="block_scale must be"):
        extensions.rms_norm_nvfp4_quant(out, scales[:100], x, w, torch.ones(1, device=DEV))
