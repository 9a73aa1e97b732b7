"""The engine-side caller (sm120_rmsnorm.engine): one attention prologue equals
the unfused sequence of the reference-API operators bit for bit, and the
captured decode graph equals eager execution."""
import pytest
import torch

import sm120_rmsnorm as ops
from numerics import assert_bitwise_equal
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
