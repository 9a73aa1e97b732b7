"""Edge cases, and the C ABI called directly through ctypes with device pointers.

Covers what the reference's suite does not: empty inputs, ragged and very
wide hidden sizes (the scalar / wide kernel families), unaligned buffers,
guard rows around outputs, out-of-range positions and slots, non-default
streams, CUDA-graph capture, and the C ABI's own argument checking. Bars as
stated in numerics.py.
"""
import ctypes

import pytest
import torch

from gpu_cases import (assert_bitwise_equal, check_norm, check_rope, expect_fused_add,
                       expect_qk, expect_rms_norm)
from sm120_rmsnorm import (capi, fused_add_rms_norm, fused_add_rms_norm_inplace,
                           fused_qk_rms_norm_rope, fused_qk_rms_norm_rope_kv, rms_norm)

pytestmark = pytest.mark.gpu
CODES = {torch.float32: capi.F32, torch.float16: capi.F16, torch.bfloat16: capi.BF16}


def rand(shape, dtype, seed=0, mean=0.0, std=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, device="cuda", generator=g) * std + mean).to(dtype)


def rope_cache(positions):
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
    freqs = torch.outer(torch.arange(positions, dtype=torch.float32, device="cuda"), inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


# ---- shapes and alignment --------------------------------------------------------

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("hidden", [1, 7, 33, 1001, 2050, 8200, 16384, 40000])
def test_ragged_and_very_wide_hidden_sizes(dtype, hidden):
    rows = 5
    x = rand((rows, hidden), dtype, hidden)
    r = rand((rows, hidden), dtype, hidden + 1)
    w = rand((hidden,), dtype, hidden + 2, 1.0, 0.1)
    check_norm(rms_norm(x, w).cpu(), expect_rms_norm(x, w), what="rms")
    expected, expected_res = expect_fused_add(x, r, w)
    out, res = fused_add_rms_norm(x, r, w)
    assert_bitwise_equal(res, expected_res, what="residual")
    check_norm(out.cpu(), expected, what="fused")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_unaligned_buffers_use_the_scalar_path(dtype):
    """Views that start one element into an allocation are not 16-byte aligned."""
    rows, hidden = 9, 1024
    base_x = rand((rows * hidden + 1,), dtype, 1)
    base_r = rand((rows * hidden + 1,), dtype, 2)
    x, r = base_x[1:].view(rows, hidden), base_r[1:].view(rows, hidden)
    w = rand((hidden,), dtype, 3, 1.0, 0.1)
    expected, expected_res = expect_fused_add(x, r, w)
    fused_add_rms_norm_inplace(x, r, w)
    assert_bitwise_equal(r, expected_res, what="residual")
    check_norm(x.cpu(), expected, what="output")
    # Q/K with a misaligned query view
    tokens = 3
    qbase = rand((tokens * 4 * 128 + 1,), dtype, 4)
    q = qbase[1:].view(tokens, 4, 128)
    k = rand((tokens, 2, 128), dtype, 5)
    qw, kw = rand((128,), dtype, 6, 1.0, 0.1), rand((128,), dtype, 7, 1.0, 0.1)
    pos = torch.tensor([5, 0, 17], device="cuda")
    cache = rope_cache(32)
    q0, k0 = q.clone(), k.clone()
    eq, ek = expect_qk(q, k, qw, kw, pos, cache)
    fused_qk_rms_norm_rope(q, k, qw, kw, pos, cache)
    check_rope(q.cpu(), eq, q0, qw, pos, cache, what="query")
    check_rope(k.cpu(), ek, k0, kw, pos, cache, what="key")


def test_guard_rows_are_untouched():
    rows, hidden = 300, 4096
    x_all = rand((rows + 2, hidden), torch.bfloat16, 8)
    r_all = rand((rows + 2, hidden), torch.bfloat16, 9)
    w = rand((hidden,), torch.bfloat16, 10, 1.0, 0.1)
    before_x, before_r = x_all.clone(), r_all.clone()
    fused_add_rms_norm_inplace(x_all[1:-1], r_all[1:-1], w)
    for i in (0, rows + 1):
        assert torch.equal(x_all[i].view(torch.int16), before_x[i].view(torch.int16))
        assert torch.equal(r_all[i].view(torch.int16), before_r[i].view(torch.int16))


def test_empty_inputs_are_no_ops():
    for dtype in (torch.bfloat16, torch.float32):
        x = torch.empty((0, 1024), device="cuda", dtype=dtype)
        w = torch.ones(1024, device="cuda", dtype=dtype)
        assert rms_norm(x, w).shape == (0, 1024)
        out, res = fused_add_rms_norm(x, x.clone(), w)
        assert out.shape == res.shape == (0, 1024)
        q = torch.empty((0, 16, 128), device="cuda", dtype=dtype)
        k = torch.empty((0, 8, 128), device="cuda", dtype=dtype)
        wq = torch.ones(128, device="cuda", dtype=dtype)
        pos = torch.empty(0, dtype=torch.int64, device="cuda")
        fused_qk_rms_norm_rope(q, k, wq, wq, pos, rope_cache(4))
        kc = torch.zeros((4, 8, 128), device="cuda", dtype=dtype)
        fused_qk_rms_norm_rope_kv(q, k, k.clone(), wq, wq, pos, rope_cache(4), kc, kc.clone(),
                                  torch.empty(0, dtype=torch.int32, device="cuda"))
        assert not kc.any()


def test_out_of_range_positions_and_slots_are_skipped():
    dtype = torch.bfloat16
    q = rand((4, 2, 128), dtype, 11)
    k = rand((4, 1, 128), dtype, 12)
    v = rand((4, 1, 128), dtype, 13)
    w = torch.ones(128, device="cuda", dtype=dtype)
    cache = rope_cache(8)
    pos = torch.tensor([0, 8, -1, 3], device="cuda")        # tokens 1, 2 out of range
    slots = torch.tensor([2, 0, 1, 4], device="cuda", dtype=torch.int32)  # slot 4 past the end
    kc = torch.zeros((4, 1, 128), device="cuda", dtype=dtype)
    vc = torch.zeros_like(kc)
    q0, k0 = q.clone(), k.clone()
    fused_qk_rms_norm_rope_kv(q, k, v, w, w, pos, cache, kc, vc, slots)
    assert torch.equal(q[1:3], q0[1:3]) and torch.equal(k[1:3], k0[1:3])
    assert not torch.equal(q[0], q0[0]) and not torch.equal(q[3], q0[3])
    assert torch.equal(kc[2], k[0]) and torch.equal(vc[2], v[0])
    kc[2].zero_()
    vc[2].zero_()
    assert not kc.any() and not vc.any()


# ---- streams and graphs ----------------------------------------------------------

def test_runs_on_the_current_stream():
    x = rand((512, 4096), torch.bfloat16, 14)
    r = rand((512, 4096), torch.bfloat16, 15)
    w = rand((4096,), torch.bfloat16, 16, 1.0, 0.1)
    expected, expected_res = expect_fused_add(x, r, w)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fused_add_rms_norm_inplace(x, r, w)
    side.synchronize()
    assert_bitwise_equal(r, expected_res, what="residual")
    check_norm(x.cpu(), expected, what="output")


def test_cuda_graph_capture_and_replay():
    x = rand((64, 2048), torch.bfloat16, 17)
    r = rand((64, 2048), torch.bfloat16, 18)
    w = rand((2048,), torch.bfloat16, 19, 1.0, 0.1)
    q = rand((64, 32, 128), torch.bfloat16, 20)
    k = rand((64, 8, 128), torch.bfloat16, 21)
    v = rand((64, 8, 128), torch.bfloat16, 22)
    qw = rand((128,), torch.bfloat16, 23, 1.0, 0.1)
    pos = torch.arange(64, device="cuda") * 5
    cache = rope_cache(512)
    kc = torch.zeros((128, 8, 128), device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.arange(64, device="cuda", dtype=torch.int32) * 2
    inputs = [t.clone() for t in (x, r, q, k, kc, vc)]

    def step():
        fused_add_rms_norm_inplace(x, r, w)
        fused_qk_rms_norm_rope_kv(q, k, v, qw, qw, pos, cache, kc, vc, slots)

    step()  # eager result
    eager = [t.clone() for t in (x, r, q, k, kc, vc)]
    for t, t0 in zip((x, r, q, k, kc, vc), inputs):
        t.copy_(t0)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for t, t0 in zip((x, r, q, k, kc, vc), inputs):
        t.copy_(t0)
    graph.replay()
    torch.cuda.synchronize()
    for got, want in zip((x, r, q, k, kc, vc), eager):
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))


# ---- the C ABI directly ----------------------------------------------------------

def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_capi_matches_the_torch_binding(dtype):
    rows, hidden = 77, 2048
    x, r = rand((rows, hidden), dtype, 30), rand((rows, hidden), dtype, 31)
    w = rand((hidden,), dtype, 32, 1.0, 0.1)
    want_out, want_res = fused_add_rms_norm(x, r, w)
    out, res = torch.empty_like(x), torch.empty_like(x)
    capi.fused_add_rms_norm(x.data_ptr(), r.data_ptr(), w.data_ptr(), out.data_ptr(),
                            res.data_ptr(), rows, hidden, CODES[dtype], 1e-6, 0, _stream())
    assert torch.equal(out, want_out) and torch.equal(res, want_res)
    y = torch.empty_like(x)
    capi.rms_norm(x.data_ptr(), w.data_ptr(), y.data_ptr(), rows, hidden, CODES[dtype], 1e-6, 2,
                  _stream())
    assert torch.equal(y, rms_norm(x, w))

    tokens = 40
    q, k, v = rand((tokens, 32, 128), dtype, 33), rand((tokens, 8, 128), dtype, 34), \
        rand((tokens, 8, 128), dtype, 35)
    qw, kw = rand((128,), dtype, 36, 1.0, 0.1), rand((128,), dtype, 37, 1.0, 0.1)
    pos = torch.arange(tokens, device="cuda") * 3
    cache = rope_cache(256)
    slots = torch.randperm(100, device="cuda")[:tokens].to(torch.int32)
    kc = torch.zeros((100, 8, 128), device="cuda", dtype=dtype)
    vc = torch.zeros_like(kc)
    q2, k2, kc2, vc2 = q.clone(), k.clone(), kc.clone(), vc.clone()
    fused_qk_rms_norm_rope_kv(q, k, v, qw, kw, pos, cache, kc, vc, slots)
    capi.fused_qk_rms_norm_rope_kv(q2.data_ptr(), k2.data_ptr(), v.data_ptr(), qw.data_ptr(),
                                   kw.data_ptr(), pos.data_ptr(), cache.data_ptr(), kc2.data_ptr(),
                                   vc2.data_ptr(), slots.data_ptr(), tokens, 32, 8, 128, 256, 100,
                                   CODES[dtype], 1e-6, 1, _stream())
    for a, b in ((q, q2), (k, k2), (kc, kc2), (vc, vc2)):
        assert torch.equal(a, b)


def test_capi_programmatic_launch_does_not_change_results():
    x, r = rand((1024, 4096), torch.bfloat16, 40), rand((1024, 4096), torch.bfloat16, 41)
    w = rand((4096,), torch.bfloat16, 42, 1.0, 0.1)
    results = []
    for enabled in (True, False):
        capi.set_programmatic_launch(enabled)
        try:
            results.append(fused_add_rms_norm(x, r, w))
        finally:
            capi.set_programmatic_launch(True)
    assert torch.equal(results[0][0], results[1][0]) and torch.equal(results[0][1], results[1][1])


def test_capi_reports_errors_without_launching():
    x = torch.zeros((4, 768), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(capi.CApiError, match="hidden_size=1024") as err:
        capi.fused_add_rms_norm(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                x.data_ptr(), 4, 768, capi.BF16, 1e-6, 3, _stream())
    assert err.value.status == capi.ERR_UNSUPPORTED
    with pytest.raises(capi.CApiError, match="head_dim=128"):
        capi.fused_qk_rms_norm_rope(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                    x.data_ptr(), x.data_ptr(), 1, 1, 1, 64, 1, capi.BF16)
    with pytest.raises(capi.CApiError, match="dtypes"):
        capi.rms_norm(x.data_ptr(), x.data_ptr(), x.data_ptr(), 4, 768, 7)
    assert not x.any()
    assert capi.device_faults() == 0
