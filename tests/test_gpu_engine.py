"""The engine-side caller (sm120_rmsnorm.engine): every layer of a captured
Qwen3-8B-shaped decode step checked against the C oracle on the layer's own
inputs; one attention prologue equals the unfused sequence of the
reference-API operators bit for bit; the captured decode graph equals eager
execution."""
import pytest
import torch

import sm120_rmsnorm as ops
from gpu_cases import check_norm, check_rope, expect_fused_add, expect_qk_kv
from numerics import assert_bitwise_equal
from sm120_rmsnorm import extensions
from sm120_rmsnorm.engine import (DecodeGraph, Qwen3AttentionPrologue, Qwen3AttentionShape,
                                  rope_cos_sin_cache)

pytestmark = pytest.mark.gpu
DEV = "cuda"
SHAPE = Qwen3AttentionShape(hidden=1024, query_heads=8, key_heads=2, max_positions=4096)


def _inputs(batch, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    hidden = torch.randn(batch, SHAPE.hidden, device=DEV, generator=g).to(torch.bfloat16)
    residual = torch.randn(batch, SHAPE.hidden, device=DEV, generator=g).to(torch.bfloat16)
    positions = torch.randint(0, SHAPE.max_positions, (batch,), device=DEV, generator=g)
    slots = torch.randperm(64 * 16, device=DEV, generator=g)[:batch].to(torch.int32)
    return hidden, residual, positions, slots


def _cache():
    return torch.zeros(64, 16, SHAPE.key_heads, SHAPE.head_dim, device=DEV, dtype=torch.bfloat16)


@pytest.mark.parametrize("batch", [1, 7, 256])
def test_prologue_equals_the_unfused_reference_api_sequence(batch):
    layer = Qwen3AttentionPrologue(SHAPE, DEV, generator=torch.Generator(device=DEV).manual_seed(1))
    cos_sin = rope_cos_sin_cache(SHAPE, DEV)
    hidden, residual, positions, slots = _inputs(batch, 2)
    h2, r2 = hidden.clone(), residual.clone()
    kc, vc = _cache(), _cache()
    qkv = torch.empty(batch, SHAPE.qkv_width, device=DEV, dtype=torch.bfloat16)
    q, k, v = layer.forward(hidden, residual, positions, cos_sin, kc, vc, slots, qkv)
    # the same layer through the reference's API: contiguous Q / K / V copies
    ops.fused_add_rms_norm_inplace(h2, r2, layer.input_norm_weight)
    qkv2 = h2 @ layer.qkv_weight.t()
    q2, k2, v2 = (t.contiguous() for t in layer.split(qkv2))
    kc2, vc2 = _cache(), _cache()
    ops.fused_qk_rms_norm_rope_kv(q2, k2, v2, layer.query_norm_weight, layer.key_norm_weight,
                                  positions, cos_sin, kc2, vc2, slots)
    assert_bitwise_equal(residual, r2, what="residual")
    assert_bitwise_equal(hidden, h2, what="normalised hidden")
    for got, want, what in ((q, q2, "query"), (k, k2, "key"), (v, v2, "value"), (kc, kc2, "key cache"),
                            (vc, vc2, "value cache")):
        assert_bitwise_equal(got.contiguous(), want, what=what)


def test_decode_graph_replays_eager_execution():
    g = torch.Generator(device=DEV).manual_seed(3)
    layers = [Qwen3AttentionPrologue(SHAPE, DEV, generator=g) for _ in range(3)]
    cos_sin = rope_cos_sin_cache(SHAPE, DEV)
    caches = [(_cache(), _cache()) for _ in layers]
    graph = DecodeGraph(layers, 5, cos_sin, [c[0] for c in caches], [c[1] for c in caches])
    hidden, residual, positions, slots = _inputs(5, 4)
    for buf, val in ((graph.hidden, hidden), (graph.residual, residual),
                     (graph.positions, positions), (graph.slot_mapping, slots)):
        buf.copy_(val)
    for kc, vc in caches:
        kc.zero_()
        vc.zero_()
    graph.replay()
    torch.cuda.synchronize()
    # eager: the same sequence on fresh buffers
    eager_caches = [(_cache(), _cache()) for _ in layers]
    h, r = hidden.clone(), residual.clone()
    for i, layer in enumerate(layers):
        qkv = torch.empty(5, SHAPE.qkv_width, device=DEV, dtype=torch.bfloat16)
        layer.forward(h, r, positions, cos_sin, eager_caches[i][0], eager_caches[i][1], slots, qkv)
        assert_bitwise_equal(graph.qkv[i], qkv, what=f"layer {i} qkv")
        assert_bitwise_equal(caches[i][0], eager_caches[i][0], what=f"layer {i} key cache")
        h = qkv[:, :SHAPE.hidden].contiguous()
    assert_bitwise_equal(graph.residual, r, what="residual after all layers")


@pytest.mark.parametrize("fused_projection", [False, True])
@pytest.mark.parametrize("batch", [1, 64])
def test_decode_graph_layers_match_the_oracle(batch, fused_projection):
    """A captured 3-layer decode step at the Qwen3-8B shape (hidden 4096, 32 / 8
    heads of 128, bf16). Per layer, from what the replay leaves behind: the
    layer's input (the previous layer's QKV buffer, or the step's input) and
    the residual carried by the oracle's own chain give the expected
    normalised hidden (1-ulp bar) and residual (bit for bit); the projection
    recomputed from the engine's normalised hidden (the same GEMM: cuBLAS, or
    this package's plain tensor-core GEMM, which the fused form is
    bit-identical to) gives the oracle's Q / K (RoPE bar), V and KV-cache
    slots (bit for bit)."""
    shape = Qwen3AttentionShape()
    g = torch.Generator(device=DEV).manual_seed(11 + batch)
    layers = [Qwen3AttentionPrologue(shape, DEV, generator=g) for _ in range(3)]
    cos_sin = rope_cos_sin_cache(shape, DEV)
    blocks = 64
    kcs = [torch.zeros(blocks, 16, shape.key_heads, 128, device=DEV, dtype=torch.bfloat16)
           for _ in layers]
    vcs = [torch.zeros_like(kc) for kc in kcs]
    graph = DecodeGraph(layers, batch, cos_sin, kcs, vcs, fused_projection=fused_projection)
    hidden0 = torch.randn(batch, shape.hidden, device=DEV, generator=g).to(torch.bfloat16)
    residual0 = torch.randn(batch, shape.hidden, device=DEV, generator=g).to(torch.bfloat16)
    positions = torch.randint(0, shape.max_positions, (batch,), device=DEV, generator=g)
    slots = torch.randperm(blocks * 16, device=DEV, generator=g)[:batch].to(torch.int32)
    for buf, val in ((graph.hidden, hidden0), (graph.residual, residual0),
                     (graph.positions, positions), (graph.slot_mapping, slots)):
        buf.copy_(val)
    for kc, vc in zip(kcs, vcs):
        kc.zero_()
        vc.zero_()
    graph.replay()
    torch.cuda.synchronize()

    residual = residual0
    hq, hk = shape.query_heads, shape.key_heads
    for i, layer in enumerate(layers):
        x_in = hidden0 if i == 0 else graph.qkv[i - 1][:, :shape.hidden].contiguous()
        normed = graph.hidden if i == 0 else graph.layer_hidden[i - 1]
        want_hidden, want_residual = expect_fused_add(x_in, residual, layer.input_norm_weight)
        check_norm(normed.cpu(), want_hidden, what=f"layer {i} normalised hidden")
        residual = want_residual.to(DEV)
        pre = torch.empty(batch, shape.qkv_width, device=DEV, dtype=torch.bfloat16)
        if fused_projection:
            extensions.qkv_proj_norm_rope_cache_(normed, layer.qkv_weight, pre, hq, hk,
                                                 fuse_norm=False)
        else:
            torch.matmul(normed, layer.qkv_weight.t(), out=pre)
        q_pre, k_pre, v_pre = (t.contiguous() for t in layer.split(pre))
        q, k, v = layer.split(graph.qkv[i])
        assert_bitwise_equal(v.contiguous(), v_pre, what=f"layer {i} value (projection)")
        small = torch.zeros(batch, 1, hk, 128, dtype=torch.bfloat16)
        want_q, want_k, want_kc, want_vc = expect_qk_kv(
            q_pre, k_pre, v_pre, layer.query_norm_weight, layer.key_norm_weight, positions,
            cos_sin, small, small.clone(), torch.arange(batch, dtype=torch.int32))
        check_rope(q.contiguous().cpu(), want_q, q_pre, layer.query_norm_weight, positions,
                   cos_sin, what=f"layer {i} query")
        check_rope(k.contiguous().cpu(), want_k, k_pre, layer.key_norm_weight, positions,
                   cos_sin, what=f"layer {i} key")
        flat_k, flat_v = kcs[i].view(-1, hk, 128), vcs[i].view(-1, hk, 128)
        assert_bitwise_equal(flat_k[slots.long()], k.contiguous(), what=f"layer {i} key cache")
        assert_bitwise_equal(flat_v[slots.long()], want_vc.view(-1, hk, 128),
                             what=f"layer {i} value cache")
    assert_bitwise_equal(graph.residual, residual, what="residual after all layers")
