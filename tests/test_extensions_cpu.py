"""CPU checks for the engine-side extensions: the extension oracle is pinned to
the reference's own oracle where the two overlap and to the e4m3fn format
definition, and the C ABI's new entry points validate their arguments (calls
that launch nothing; no GPU needed)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import extensions as ex
from oracle import oracle
from sm120_rmsnorm import capi
from sm120_rmsnorm.reference import (
    fused_add_rms_norm_reference,
    qk_rms_norm_rope_reference,
    rms_norm_reference,
)

from numerics import assert_bitwise_equal, assert_rope_close, assert_ulp_close, rope_bound


def _cache_table(positions, rotary, base=1e6):
    inv = 1.0 / (base ** (torch.arange(0, rotary, 2, dtype=torch.float32) / rotary))
    f = torch.outer(torch.arange(positions, dtype=torch.float32), inv)
    return torch.cat((f.cos(), f.sin()), dim=-1)


# ---- fp8 e4m3fn conversion ---------------------------------------------------------
def test_e4m3_decode_matches_torch_for_every_code():
    codes = torch.arange(256, dtype=torch.uint8)
    mine = np.array([ex.e4m3_decode(c) for c in range(256)])
    theirs = codes.view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(mine), np.isnan(theirs))
    finite = ~np.isnan(mine)
    assert np.array_equal(mine[finite], theirs[finite])
    assert np.nanmax(mine) == 448.0


def test_e4m3_saturating_conversion_matches_the_format_definition():
    g = torch.Generator().manual_seed(3)
    table = np.array([ex.e4m3_decode(c) for c in range(256)])
    finite = np.sort(np.unique(table[~np.isnan(table)]))
    mids = (finite[1:] + finite[:-1]) / 2  # exact ties
    probes = [
        finite, mids, np.nextafter(mids, np.inf), np.nextafter(mids, -np.inf),
        np.array([0.0, -0.0, 448.0, 449.0, 463.9, 464.0, 465.0, 1e6, -1e6, 2.0 ** -10,
                  -(2.0 ** -10), 2.0 ** -11, 3 * 2.0 ** -11]),
        (torch.randn(4000, generator=g) * torch.pow(2.0, torch.randint(-12, 10, (4000,),
                                                                      generator=g))).numpy(),
    ]
    values = np.concatenate(probes).astype(np.float32)
    got = ex.fp8_e4m3(torch.from_numpy(values)).view(torch.uint8).numpy()
    want = ex.e4m3_round_reference(values)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, (values[bad[:5]], got[bad[:5]], want[bad[:5]])


# ---- generalised Q/K oracle against the reference's oracle ---------------------------
def exact_values(shape, dtype, g, limit=32):
    """k / 16 for integer k in [-limit, limit]: sums of squares exact in fp32."""
    return (torch.randint(-limit, limit + 1, shape, generator=g).float() / 16).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_generalised_oracle_equals_the_reference_oracle_at_head_dim_128(dtype):
    g = torch.Generator().manual_seed(11)
    tokens, hq, hk = 9, 4, 2
    q = exact_values((tokens, hq, 128), dtype, g)
    k = exact_values((tokens, hk, 128), dtype, g)
    v = exact_values((tokens, hk, 128), dtype, g)
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(dtype)
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(dtype)
    table = _cache_table(64, 128)
    pos = torch.randint(0, 64, (tokens,), generator=g)
    slots = torch.randperm(4 * 16, generator=g)[:tokens].to(torch.int32)
    kc = torch.zeros(4, 16, hk, 128, dtype=dtype)
    gq, gk, gkc, gvc = ex.qk_norm_rope_cache(q, k, v, qw, kw, pos, table, kc, kc.clone(), slots)
    # the C restatement of the reference's KV variant: the same IEEE
    # evaluation, so with exact sums of squares every bit agrees
    cq, ck, ckc, cvc = q.clone(), k.clone(), kc.clone(), kc.clone()
    oracle.build()
    oracle.qk_rms_norm_rope_kv_(cq, ck, v, qw, kw, pos, table, ckc, cvc, slots)
    for got, want, what in ((gq, cq, "query"), (gk, ck, "key"), (gkc, ckc, "key cache"),
                            (gvc, cvc, "value cache")):
        assert_bitwise_equal(got, want, what=f"{what} vs C oracle")
    # the reference's PyTorch oracle (its CPU rsqrt is not IEEE on every
    # build): within the propagated RoPE bar
    rq, rk = qk_rms_norm_rope_reference(q, k, qw, kw, pos, table.unsqueeze(1))
    assert_rope_close(gq, rq, rope_bound(q, qw, pos, table, rq), what="query vs reference.py")
    assert_rope_close(gk, rk, rope_bound(k, kw, pos, table, rk), what="key vs reference.py")


def test_interleaved_and_partial_rotary_follow_their_definitions():
    g = torch.Generator().manual_seed(5)
    tokens, heads, d, rotary = 3, 2, 64, 32
    x = torch.randn(tokens, heads, d, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    table = _cache_table(16, rotary)
    pos = torch.tensor([0, 5, 15])
    for neox in (True, False):
        got, _, _, _ = ex.qk_norm_rope_cache(x, x[:, :0], None, w, w, pos, table, is_neox=neox)
        n = (torch.nn.functional.rms_norm(x.float(), (d,), None, 1e-6).to(torch.bfloat16) * w)
        for t in range(tokens):
            c, s = table[pos[t], :rotary // 2], table[pos[t], rotary // 2:]
            for h in range(heads):
                row = n[t, h].float()
                want = row.clone()
                for i in range(rotary // 2):
                    a, b = (i, i + rotary // 2) if neox else (2 * i, 2 * i + 1)
                    want[a] = row[a] * c[i] - row[b] * s[i]
                    want[b] = row[b] * c[i] + row[a] * s[i]
                want = want.to(torch.bfloat16)
                want[rotary:] = n[t, h, rotary:]
                assert_bitwise_equal(got[t, h], want, what=f"neox={neox} t={t} h={h}")


def test_hnd_cache_is_the_nhd_cache_transposed():
    g = torch.Generator().manual_seed(8)
    tokens, hk = 7, 3
    q = torch.randn(tokens, 2, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(tokens, hk, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(tokens, hk, 64, generator=g).to(torch.bfloat16)
    w = torch.ones(64, dtype=torch.bfloat16)
    table = _cache_table(32, 64)
    pos = torch.randint(0, 32, (tokens,), generator=g)
    slots = torch.tensor([3, -1, 40, 9, 17, 100, 0], dtype=torch.int32)  # 100 is outside
    nhd = torch.zeros(3, 16, hk, 64, dtype=torch.bfloat16)
    hnd = torch.zeros(3, hk, 16, 64, dtype=torch.bfloat16)
    _, _, a, _ = ex.qk_norm_rope_cache(q, k, v, w, w, pos, table, nhd, nhd.clone(), slots)
    _, _, b, _ = ex.qk_norm_rope_cache(q, k, v, w, w, pos, table, hnd, hnd.clone(), slots,
                                       kv_cache_layout="HND")
    assert_bitwise_equal(a, b.transpose(1, 2), what="HND vs NHD")
    assert int((a != 0).any(-1).any(-1).sum()) == 5  # -1 and 100 (>= 48 slots) skipped


def test_fp8_cache_store_divides_by_the_scale():
    g = torch.Generator().manual_seed(9)
    k = torch.randn(2, 1, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(2, 1, 64, generator=g).to(torch.bfloat16) * 300
    w = torch.ones(64, dtype=torch.bfloat16)
    table = _cache_table(4, 64)
    pos = torch.tensor([1, 2])
    slots = torch.tensor([0, 1], dtype=torch.int32)
    cache = torch.zeros(1, 2, 1, 64, dtype=torch.uint8)
    ks, vs = torch.tensor([0.5]), torch.tensor([0.25])
    _, kk, kc, vc = ex.qk_norm_rope_cache(k[:, :0], k, v, w, w, pos, table, cache, cache.clone(),
                                          slots, ks, vs)
    want_k = ex.e4m3_round_reference((kk.float() / 0.5).numpy())
    want_v = ex.e4m3_round_reference((v.float() / 0.25).numpy())
    assert np.array_equal(kc[0].numpy(), want_k)
    assert np.array_equal(vc[0].numpy(), want_v)  # saturates: |v| / 0.25 exceeds 448


# ---- RMSNorm + fp8 oracle ------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_norm_rows_equal_the_reference_oracle(dtype):
    g = torch.Generator().manual_seed(2)
    x = exact_values((5, 768), dtype, g, limit=8)
    r = exact_values((5, 768), dtype, g, limit=8)
    w = (1 + 0.1 * torch.randn(768, generator=g)).to(dtype)
    oracle.build()
    y, _ = ex.rms_norm_rows(x, w)
    assert_bitwise_equal(y, oracle.rms_norm(x, w, 1e-6), what="rms_norm vs C oracle")
    assert_ulp_close(y, rms_norm_reference(x, w), what="rms_norm vs reference.py")
    y, s = ex.rms_norm_rows(x, w, residual=r)
    want_y, want_s = oracle.fused_add_rms_norm(x, r, w, 1e-6)
    assert_bitwise_equal(y, want_y, what="fused output vs C oracle")
    assert_bitwise_equal(s, want_s, what="fused residual vs C oracle")
    ref_y, ref_s = fused_add_rms_norm_reference(x, r, w)
    assert_ulp_close(y, ref_y, what="fused output vs reference.py")
    assert_bitwise_equal(s, ref_s, what="fused residual vs reference.py")


def test_dynamic_scales_follow_their_definition():
    y = torch.tensor([[1.0, -3.0, 2.0], [0.0, 0.0, 0.0], [900.0, 1.0, -2.0]]).to(torch.bfloat16)
    q, scales = ex.quantise_rows(y)
    assert scales[0].item() == np.float32(3.0) / np.float32(448.0)
    assert scales[1].item() == ex.MIN_TOKEN_SCALE  # all-zero row: the floor
    assert q[0].float().abs().max().item() == 448.0
    q_ub, scales_ub = ex.quantise_rows(y, scale_ub=torch.tensor([10.0]))
    assert scales_ub[2].item() == np.float32(10.0) / np.float32(448.0)
    assert q_ub[2, 0].float().item() == 448.0  # saturated by the bound


# ---- C ABI of the extensions (argument checks only: nothing is launched) -----------------
def test_extension_symbols_are_exported():
    lib = ctypes.CDLL(str(capi.LIBRARY_PATH))
    for name in ("sm120n_qk_norm_rope_cache", "sm120n_rms_norm_fp8_quant"):
        assert hasattr(lib, name)


def test_qk_cache_struct_layout_matches_the_library():
    args = capi.QkCacheArgs(dtype=capi.BF16, tokens=0, query_heads=1, key_heads=1, head_dim=128,
                            rotary_dim=128)
    capi.qk_norm_rope_cache(args)  # zero tokens: validated and accepted
    args.struct_size = ctypes.sizeof(capi.QkCacheArgs) - 8
    with pytest.raises(capi.CApiError, match="struct_size"):
        capi.qk_norm_rope_cache(args)


@pytest.mark.parametrize("field, value, message", [
    ("head_dim", 96, "head_dim must be 64, 128 or 256"),
    ("rotary_dim", 24, "rotary_dim must be a multiple of 16"),
    ("rotary_dim", 256, "rotary_dim must be a multiple of 16"),
    ("rope_style", 7, "unknown rope_style"),
    ("cache_dtype", 9, "unknown cache_dtype"),
    ("dtype", 5, "supported dtypes"),
    ("tokens", -1, "non-negative"),
])
def test_qk_cache_rejects_bad_arguments(field, value, message):
    args = capi.QkCacheArgs(dtype=capi.BF16, tokens=0, query_heads=1, key_heads=1, head_dim=128,
                            rotary_dim=128)
    setattr(args, field, value)
    with pytest.raises(capi.CApiError, match=message):
        capi.qk_norm_rope_cache(args)


def test_qk_cache_rejects_overlapping_token_rows_and_missing_scales():
    args = capi.QkCacheArgs(dtype=capi.BF16, tokens=4, query_heads=2, key_heads=1, head_dim=64,
                            rotary_dim=64, query=16, query_token_stride=64, key=16,
                            key_token_stride=64, query_weight=16, key_weight=16, positions=16,
                            cos_sin_cache=16)
    with pytest.raises(capi.CApiError, match="token strides"):
        capi.qk_norm_rope_cache(args)
    args.query_token_stride = 128
    args.key_cache, args.value_cache, args.value, args.slot_mapping = 16, 16, 16, 16
    args.value_token_stride, args.num_blocks, args.block_size = 64, 1, 16
    args.cache_dtype = capi.CACHE_FP8_E4M3
    with pytest.raises(capi.CApiError, match="k_scale and v_scale"):
        capi.qk_norm_rope_cache(args)


def test_norm_quant_rejects_bad_arguments():
    with pytest.raises(capi.CApiError, match="exactly one of scale"):
        capi.rms_norm_fp8_quant(16, None, 16, None, 16, None, None, None, 1, 64, capi.BF16)
    with pytest.raises(capi.CApiError, match="exactly one of scale"):
        capi.rms_norm_fp8_quant(16, None, 16, None, 16, 16, 16, None, 1, 64, capi.BF16)
    with pytest.raises(capi.CApiError, match="scale_ub applies to dynamic"):
        capi.rms_norm_fp8_quant(16, None, 16, None, 16, 16, None, 16, 1, 64, capi.BF16)
    with pytest.raises(capi.CApiError, match="residual and residual_output go together"):
        capi.rms_norm_fp8_quant(16, 16, 16, None, 16, 16, None, None, 1, 64, capi.BF16)
    with pytest.raises(capi.CApiError, match="hidden_size"):
        capi.rms_norm_fp8_quant(16, None, 16, None, 16, 16, None, None, 1, 0, capi.BF16)
    capi.rms_norm_fp8_quant(0, None, 0, None, 0, 16, None, None, 0, 64, capi.BF16)  # no rows


# ---- NVFP4 ------------------------------------------------------------------------
def test_e2m1_rounding_follows_the_format_definition():
    values = np.array([0, 0.24, 0.25, 0.26, 0.75, 1.25, 1.75, 2.5, 3.5, 5, 5.1, 7, 100,
                       -0.1, -0.0, -5, -0.75], dtype=np.float32)
    # ties go to the even code: 0.25 -> 0, 0.75 -> 1.0, 1.25 -> 1.0, 1.75 -> 2,
    # 2.5 -> 2, 3.5 -> 4, 5 -> 4; beyond 6 saturates; the sign bit is kept
    want = [0, 0, 0, 1, 2, 2, 4, 4, 6, 6, 7, 7, 7, 8, 8, 14, 10]
    assert ex.e2m1_codes(values).tolist() == want
    decoded = ex.E2M1_MAGNITUDES[np.array(want) & 7]
    assert decoded.max() == 6.0


def test_tiled_scale_layout_is_the_128x4_block_interleave():
    rows, blocks = 300, 10
    offsets = ex.nvfp4_scale_offsets(rows, blocks, tiled=True)
    # restated as a reshape: pad to (384, 12), view (tiles_m, 4, 32, tiles_k, 4),
    # order the axes (tiles_m, tiles_k, 32, 4, 4)
    padded = torch.full((384, 12), -1, dtype=torch.int64)
    padded[:rows, :blocks] = torch.arange(rows * blocks).reshape(rows, blocks)
    order = padded.reshape(3, 4, 32, 3, 4).permute(0, 3, 2, 1, 4).reshape(-1)
    position = torch.empty(rows * blocks, dtype=torch.int64)
    real = order >= 0
    position[order[real]] = torch.nonzero(real).flatten()
    assert np.array_equal(offsets.reshape(-1), position.numpy())
    assert np.array_equal(ex.nvfp4_scale_offsets(rows, blocks, tiled=False).reshape(-1),
                          np.arange(rows * blocks))


def test_nvfp4_block_scales_and_values():
    y = torch.zeros(1, 32, dtype=torch.bfloat16)
    y[0, :16] = torch.tensor([3.0, -1.5, 0.0] + [0.25] * 13)
    y[0, 16:] = 0.0  # an all-zero block: scale 0, values 0
    packed, scales = ex.nvfp4_quantise(y, 2.0, tiled=False)
    # block 0: peak 3, s = e4m3(2 * (3 * fp32(1/6))) = 1.0, r = g / s = 2: y * 2
    assert scales.tolist() == [0x38, 0x00]  # 1.0 in e4m3 is 0x38
    codes = np.stack([packed.numpy() & 0xF, packed.numpy() >> 4], -1).reshape(-1)
    assert codes[:4].tolist() == [7, 13, 0, 1]  # 6, -3 (sign | code 5), 0, 0.5
    assert codes[16:].tolist() == [0] * 16


def test_fp4_quant_rejects_bad_arguments():
    with pytest.raises(capi.CApiError, match="multiple of 16"):
        capi.rms_norm_fp4_quant(16, None, 16, None, 16, 16, 16, 1, 72, capi.BF16)
    with pytest.raises(capi.CApiError, match="unknown scale_layout"):
        capi.rms_norm_fp4_quant(16, None, 16, None, 16, 16, 16, 1, 64, capi.BF16,
                                scale_layout=5)
    with pytest.raises(capi.CApiError, match="residual and residual_output go together"):
        capi.rms_norm_fp4_quant(16, 16, 16, None, 16, 16, 16, 1, 64, capi.BF16)
    with pytest.raises(capi.CApiError, match="16-byte-aligned"):
        capi.rms_norm_fp4_quant(8, None, 16, None, 16, 16, 16, 1, 64, capi.BF16)
    with pytest.raises(capi.CApiError, match="must be non-null"):
        capi.rms_norm_fp4_quant(16, None, 16, None, 16, None, 16, 1, 64, capi.BF16)
    capi.rms_norm_fp4_quant(0, None, 0, None, 0, 0, 0, 0, 64, capi.BF16)  # no rows
