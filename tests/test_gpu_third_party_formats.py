"""The engine-side data formats pinned to an independent implementation that
is installed here: vLLM's own CUDA kernels (used only as a checker).

  * fp8 e4m3 KV cache: the bytes this package stores for the rotated K and
    for V equal those of vLLM's reshape_and_cache_flash (kv_cache_dtype
    "fp8") given the same rotated K, V, slots and k / v scales -- including
    scales small enough to saturate;
  * NVFP4: the e2m1 codes and e4m3 block scales of rms_norm_nvfp4_quant, in
    the 128 x 4 tiled scale layout, equal those of vLLM's scaled_fp4_quant
    (swizzled scales) of the same normalised rows. On exact-sum inputs the
    normalised rows are unique, so codes and scales must agree bit for bit;
    on random inputs the differences are counted and printed, and each one
    must be a single step of the format.

Skipped when vLLM's kernels do not load in this process."""
import importlib.util
from pathlib import Path

import pytest
import torch

from oracle.extensions import nvfp4_scale_offsets
from sm120_rmsnorm import extensions as ext
from sm120_rmsnorm import rms_norm

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _vllm():
    spec = importlib.util.find_spec("vllm")
    if spec is None or not spec.submodule_search_locations:
        return None
    root = Path(list(spec.submodule_search_locations)[0])
    try:
        for name in ("_C.abi3.so", "_C_stable_libtorch.abi3.so"):
            torch.ops.load_library(str(root / name))
        return torch.ops._C, torch.ops._C_cache_ops
    except Exception:  # noqa: BLE001 - the checker is optional
        return None


VLLM = _vllm() if torch.cuda.is_available() else None
needs_vllm = pytest.mark.skipif(VLLM is None, reason="vLLM's kernels do not load here")


def _rope_table(n):
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device=DEV) / 128))
    f = torch.outer(torch.arange(n, dtype=torch.float32, device=DEV), inv)
    return torch.cat((f.cos(), f.sin()), dim=-1)


@needs_vllm
@pytest.mark.parametrize("k_scale,v_scale", [(0.05, 0.1), (0.004, 0.003), (1.0, 1.0)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_kv_cache_bytes_match_vllm(k_scale, v_scale, dtype):
    _, cache_ops = VLLM
    g = torch.Generator(device=DEV).manual_seed(7)
    tokens, hq, hk, blocks = 256, 32, 8, 64
    q = torch.randn(tokens, hq, 128, device=DEV, generator=g).to(dtype)
    k = torch.randn(tokens, hk, 128, device=DEV, generator=g).to(dtype)
    v = (3 * torch.randn(tokens, hk, 128, device=DEV, generator=g)).to(dtype)
    qw = (1 + 0.1 * torch.randn(128, device=DEV, generator=g)).to(dtype)
    kw = (1 + 0.1 * torch.randn(128, device=DEV, generator=g)).to(dtype)
    pos = torch.randint(0, 4096, (tokens,), device=DEV, generator=g)
    slots = torch.randperm(blocks * 16, device=DEV, generator=g)[:tokens].to(torch.int32)
    ks = torch.tensor([k_scale], device=DEV)
    vs = torch.tensor([v_scale], device=DEV)
    kc = torch.zeros(blocks, 16, hk, 128, device=DEV, dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    ext.qk_norm_rope_cache_(q, k, v, qw, kw, pos, _rope_table(4096), kc, vc, slots, ks, vs)
    # k now holds the rotated K this package stored; vLLM stores the same K and V
    vkc = torch.zeros(blocks, 16, hk, 128, device=DEV, dtype=torch.uint8)
    vvc = torch.zeros_like(vkc)
    cache_ops.reshape_and_cache_flash(k, v, vkc, vvc, slots.long(), "fp8", ks, vs)
    torch.cuda.synchronize()
    assert torch.equal(kc.view(torch.uint8), vkc), \
        f"{int((kc.view(torch.uint8) != vkc).sum())} key-cache bytes differ from vLLM's"
    assert torch.equal(vc.view(torch.uint8), vvc), \
        f"{int((vc.view(torch.uint8) != vvc).sum())} value-cache bytes differ from vLLM's"


def _exact_values(shape, dtype, g, limit):
    """Multiples of 1/16 in [-limit, limit]: every square and partial sum of
    squares is exact in fp32, so the normalised rows do not depend on the
    summation order."""
    return (torch.randint(-16 * limit, 16 * limit + 1, shape, device=DEV, generator=g)
            .to(torch.float32) / 16).to(dtype)


def _vllm_fp4(y, gscale):
    C, _ = VLLM
    rows, hidden = y.shape
    q = torch.empty(rows, hidden // 2, device=DEV, dtype=torch.uint8)
    scales = torch.zeros(ext.nvfp4_scale_bytes(rows, hidden) // 4, device=DEV, dtype=torch.int32)
    C.scaled_fp4_quant.out(y, gscale, True, output=q, output_scale=scales)
    return q, scales.view(torch.uint8)


def _ours_fp4(x, w, gscale, residual=None):
    rows, hidden = x.shape
    q = torch.empty(rows, hidden // 2, device=DEV, dtype=torch.uint8)
    scales = torch.zeros(ext.nvfp4_scale_bytes(rows, hidden), device=DEV, dtype=torch.uint8)
    ext.rms_norm_nvfp4_quant(q, scales, x, w, gscale, 1e-6, residual, True)
    return q, scales


def _real_scales(scales, rows, hidden):
    """The scale bytes of real (row, block) pairs, in row-major order (the
    tiled layout's padding rows and columns are left out)."""
    offsets = torch.from_numpy(nvfp4_scale_offsets(rows, hidden // 16, True)).reshape(-1)
    return scales.cpu()[offsets]


def _e2m1_steps(a, b):
    def nibbles(t):
        t = t.to(torch.int16)
        codes = torch.stack((t & 0xF, t >> 4), -1)
        return torch.where(codes >= 8, -(codes & 7), codes)
    return (nibbles(a) - nibbles(b)).abs()


@needs_vllm
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,hidden", [(256, 4096), (200, 8192), (1200, 8192)])
@pytest.mark.parametrize("add", [False, True])
def test_nvfp4_codes_and_tiled_scales_match_vllm_exact_inputs(dtype, rows, hidden, add):
    g = torch.Generator(device=DEV).manual_seed(rows + hidden + add)
    limit = 8 if add else 16
    x = _exact_values((rows, hidden), dtype, g, limit)
    r = _exact_values((rows, hidden), dtype, g, limit) if add else None
    w = (torch.randint(12, 21, (hidden,), device=DEV, generator=g).to(torch.float32) / 16).to(dtype)
    gscale = torch.tensor([448.0 * 6.0 / 5.0], device=DEV)
    summed = x + r if add else x
    y = rms_norm(summed, w)  # the rows this package quantises (unique on exact inputs)
    want_q, want_scales = _vllm_fp4(y, gscale)
    q, scales = _ours_fp4(x, w, gscale, r.clone() if add else None)
    torch.cuda.synchronize()
    scales, want_scales = (_real_scales(s, rows, hidden) for s in (scales, want_scales))
    assert torch.equal(scales, want_scales), \
        f"{int((scales != want_scales).sum())} block-scale bytes differ from vLLM's"
    assert torch.equal(q, want_q), f"{int((q != want_q).sum())} code bytes differ from vLLM's"


@needs_vllm
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_nvfp4_random_rows_against_vllm(dtype):
    """Random N(0,1) rows: vLLM quantises this package's RMSNorm output; the
    NVFP4 operator quantises its own normalised rows (the same values except
    where a different fp32 summation order moves an element by one ulp), so
    differences are counted, printed and must be one format step each."""
    g = torch.Generator(device=DEV).manual_seed(31)
    rows, hidden = 1024, 4096
    x = torch.randn(rows, hidden, device=DEV, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, device=DEV, generator=g)).to(dtype)
    gscale = torch.tensor([448.0 * 6.0 / 5.0], device=DEV)
    want_q, want_scales = _vllm_fp4(rms_norm(x, w), gscale)
    q, scales = _ours_fp4(x, w, gscale)
    torch.cuda.synchronize()
    scales, want_scales = (_real_scales(s, rows, hidden) for s in (scales, want_scales))
    scale_diff = int((scales != want_scales).sum())
    steps = _e2m1_steps(q.cpu(), want_q.cpu())
    code_diff = int((steps > 0).sum())
    print(f"NVFP4 {dtype}: {scale_diff} of {scales.numel()} scale bytes and {code_diff} of "
          f"{steps.numel()} codes differ from vLLM's")
    assert scale_diff <= 1e-3 * scales.numel()
    assert int(steps.max()) <= 1
    assert code_diff <= 1e-3 * steps.numel()
