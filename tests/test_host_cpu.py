"""Host-side checks that need no GPU: the C-ABI library and its exports, the
C ABI's argument checking, the torch binding's error messages and schemas,
and the loud failure of the operators when the extension is missing."""
import re
from pathlib import Path

import pytest
import torch

import sm120_rmsnorm
from sm120_rmsnorm import capi, ops

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "sm120norm_b200.h"


def header_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"SM120N_API\s+[\w\s\*]+?\b(sm120n_\w+)\s*\(", text))


def test_library_loads_and_exports_every_declared_symbol():
    lib = capi.load()
    declared = header_symbols()
    assert len(declared) == 17, declared
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(capi.SIGNATURES), "capi.SIGNATURES must bind exactly the header"
    assert capi.abi_version() == 5


def test_library_exports_nothing_else():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIBRARY_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == header_symbols()


def test_status_strings():
    lib = capi.load()
    assert lib.sm120n_status_string(0) == b"ok"
    assert lib.sm120n_status_string(2) == b"unsupported"


@pytest.mark.parametrize("call, status, message", [
    (lambda: capi.rms_norm(0, 0, 0, 4, 1024, capi.BF16, 1e-6, 3), capi.ERR_INVALID_ARGUMENT,
     "RMSNorm version must be 1 or 2"),
    (lambda: capi.rms_norm(0, 0, 0, 4, 1024, 9), capi.ERR_INVALID_ARGUMENT, "supported dtypes"),
    (lambda: capi.rms_norm(0, 0, 0, -1, 1024, capi.BF16), capi.ERR_INVALID_ARGUMENT, "rows"),
    (lambda: capi.rms_norm(0, 0, 0, 4, 1024, capi.BF16), capi.ERR_INVALID_ARGUMENT, "non-null"),
    (lambda: capi.fused_add_rms_norm(0, 0, 0, 0, 0, 4, 768, capi.F16, 1e-6, 3),
     capi.ERR_UNSUPPORTED, "V3 is specialized for hidden_size=1024"),
    (lambda: capi.fused_add_rms_norm(0, 0, 0, 0, 0, 4, 768, capi.F16, 1e-6, 1),
     capi.ERR_INVALID_ARGUMENT, "fused version must be 0 (auto), 2, 3, or 4"),
    (lambda: capi.fused_qk_rms_norm_rope(0, 0, 0, 0, 0, 0, 1, 16, 8, 64, 8, capi.BF16),
     capi.ERR_UNSUPPORTED, "fused QK Norm+RoPE requires head_dim=128"),
    (lambda: capi.fused_qk_rms_norm_rope(0, 0, 0, 0, 0, 0, 1, 16, 8, 128, 8, capi.BF16, 1e-6, 3),
     capi.ERR_INVALID_ARGUMENT, "QK Norm+RoPE version must be 1 or 2"),
    (lambda: capi.fused_qk_rms_norm_rope_kv(0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 16, 8, 96, 8, 4,
                                            capi.BF16), capi.ERR_UNSUPPORTED,
     "fused QK Norm+RoPE+KV requires head_dim=128"),
    (lambda: capi.fused_qk_rms_norm_rope_kv(0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 16, 8, 128, 8, 4,
                                            capi.BF16, 1e-6, 2), capi.ERR_INVALID_ARGUMENT,
     "QK Norm+RoPE+KV version must be 1 or 4 warps per block"),
])
def test_capi_argument_checking(call, status, message):
    with pytest.raises(capi.CApiError) as err:
        call()
    assert err.value.status == status
    assert message in str(err.value)


def test_capi_empty_inputs_need_no_device():
    capi.rms_norm(0, 0, 0, 0, 1024, capi.BF16)
    capi.fused_add_rms_norm(0, 0, 0, 0, 0, 0, 1024, capi.BF16)
    capi.fused_qk_rms_norm_rope(0, 0, 0, 0, 0, 0, 0, 16, 8, 128, 8, capi.BF16)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks behaviour without a GPU")
def test_capi_fails_loudly_without_a_device():
    buf = torch.zeros(64)
    with pytest.raises(capi.CApiError) as err:
        capi.rms_norm(buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), 1, 16, capi.F32)
    assert err.value.status == capi.ERR_CUDA


def test_binding_rejects_host_tensors_with_the_reference_messages():
    x = torch.randn(4, 1024, dtype=torch.bfloat16)
    w = torch.randn(1024, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="input must be a CUDA tensor"):
        sm120_rmsnorm.rms_norm(x, w)
    with pytest.raises(RuntimeError, match="input must be a CUDA tensor"):
        sm120_rmsnorm.fused_add_rms_norm_inplace(x, x.clone(), w)
    with pytest.raises(RuntimeError, match="Q/K/V must be CUDA tensors"):
        ops._C.fused_qk_rms_norm_rope_kv(
            torch.randn(1, 16, 128), torch.randn(1, 8, 128), torch.randn(1, 8, 128),
            torch.ones(128), torch.ones(128), torch.zeros(1, dtype=torch.long),
            torch.zeros(4, 128), torch.zeros(4, 8, 128), torch.zeros(4, 8, 128),
            torch.zeros(1, dtype=torch.int32), 1e-6, 1)


def test_torch_library_schemas_match_the_reference():
    schemas = {
        "fused_qk_rms_norm_rope_": (
            "sm120_norm::fused_qk_rms_norm_rope_(Tensor(a!) query, Tensor(b!) key, "
            "Tensor query_weight, Tensor key_weight, Tensor positions, Tensor cos_sin_cache, "
            "float epsilon=9.9999999999999995e-07, int version=2) -> ()"),
        "fused_qk_rms_norm_rope_kv_": (
            "sm120_norm::fused_qk_rms_norm_rope_kv_(Tensor(a!) query, Tensor(b!) key, "
            "Tensor value, Tensor query_weight, Tensor key_weight, Tensor positions, "
            "Tensor cos_sin_cache, Tensor(c!) key_cache, Tensor(d!) value_cache, "
            "Tensor slot_mapping, float epsilon=9.9999999999999995e-07, int version=1) -> ()"),
    }
    for name, schema in schemas.items():
        assert str(getattr(torch.ops.sm120_norm, name).default._schema) == schema


def test_public_api_matches_the_reference_names_and_defaults():
    import inspect
    expected = {
        "rms_norm": ["x", "weight", "epsilon", "version"],
        "rms_norm_out": ["x", "weight", "output", "epsilon", "version"],
        "fused_add_rms_norm": ["x", "residual", "weight", "epsilon", "version"],
        "fused_add_rms_norm_out": ["x", "residual", "weight", "output", "residual_output",
                                   "epsilon", "version"],
        "fused_add_rms_norm_inplace": ["x", "residual", "weight", "epsilon", "version"],
        "fused_qk_rms_norm_rope": ["query", "key", "query_weight", "key_weight", "positions",
                                   "cos_sin_cache", "epsilon", "version"],
        "fused_qk_rms_norm_rope_kv": ["query", "key", "value", "query_weight", "key_weight",
                                      "positions", "cos_sin_cache", "key_cache", "value_cache",
                                      "slot_mapping", "epsilon", "version"],
    }
    defaults = {"rms_norm": 2, "rms_norm_out": 2, "fused_add_rms_norm": 0,
                "fused_add_rms_norm_out": 0, "fused_add_rms_norm_inplace": 0,
                "fused_qk_rms_norm_rope": 2, "fused_qk_rms_norm_rope_kv": 1}
    for name, params in expected.items():
        sig = inspect.signature(getattr(sm120_rmsnorm, name))
        assert list(sig.parameters) == params, name
        assert sig.parameters["epsilon"].default == 1e-6
        assert sig.parameters["version"].default == defaults[name]
    assert set(sm120_rmsnorm.__all__) >= set(expected) | {
        "rms_norm_reference", "fused_add_rms_norm_reference", "qk_rms_norm_rope_reference"}


def test_operators_fail_loudly_without_the_extension(monkeypatch):
    monkeypatch.setattr(ops, "_C", None)
    x = torch.randn(2, 8)
    with pytest.raises(RuntimeError, match="extension is not built"):
        ops.rms_norm(x, torch.ones(8))
    with pytest.raises(RuntimeError, match="extension is not built"):
        ops.fused_qk_rms_norm_rope(x, x, x, x, x, x)


def test_reference_exports_match_the_oracle_on_cpu():
    """The exported *_reference functions and the C oracle agree (both restate
    the same math)."""
    from oracle import oracle
    from numerics import assert_ulp_close
    oracle.build()
    torch.manual_seed(0)
    x = torch.randn(33, 2048).to(torch.bfloat16)
    r = torch.randn(33, 2048).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(2048)).to(torch.bfloat16)
    a, b = sm120_rmsnorm.fused_add_rms_norm_reference(x, r, w)
    c, d = oracle.fused_add_rms_norm(x, r, w)
    assert torch.equal(b, d)
    assert_ulp_close(c, a)


def test_fp32_norm_bar_grows_with_the_row_length():
    """The fp32 norm bar: 4 ulp up to 1024 elements, 4 * ceil(sqrt(n / 1024))
    beyond; 16-bit outputs keep 1 ulp at every length."""
    from numerics import default_norm_ulps
    assert [default_norm_ulps(torch.float32, n) for n in (1, 1024, 1025, 2560, 4096, 8192)] == \
        [4, 4, 8, 8, 8, 12]
    assert default_norm_ulps(torch.bfloat16, 8192) == 1 and default_norm_ulps(torch.float16, 8192) == 1


@pytest.mark.parametrize("hidden", [1024, 2560, 8192])
def test_fp32_bar_covers_two_summation_orders(hidden):
    """Two CPU restatements that add the squares in different fp32 orders (the
    C oracle's lane tree and PyTorch's reduction) stay within the bar."""
    from oracle import oracle
    from numerics import assert_ulp_close
    oracle.build()
    g = torch.Generator().manual_seed(hidden)
    x = torch.randn(64, hidden, generator=g)
    w = 1 + 0.1 * torch.randn(hidden, generator=g)
    assert_ulp_close(oracle.rms_norm(x, w), sm120_rmsnorm.rms_norm_reference(x, w), what="fp32 rms_norm")


def test_wait_limit_setting_clamps_and_restores():
    default = capi.wait_limit()
    assert default == 1 << 22
    try:
        capi.set_wait_limit(3)
        assert capi.wait_limit() == 3
        capi.set_wait_limit(1 << 30)  # above the default: clamped to it
        assert capi.wait_limit() == default
        capi.set_wait_limit(5)
        capi.set_wait_limit(0)  # 0 restores the default
        assert capi.wait_limit() == default
    finally:
        capi.set_wait_limit(0)


def test_engine_picks_the_fused_projection_only_where_it_pays():
    from sm120_rmsnorm.engine import DecodeGraph, Qwen3AttentionShape

    shape = Qwen3AttentionShape()
    bf16_caches = [torch.zeros(4, 16, 8, 128, dtype=torch.bfloat16)]
    pays = DecodeGraph.fused_projection_pays
    assert pays(1, shape, torch.bfloat16, bf16_caches, None, "NHD")
    assert pays(4, shape, torch.bfloat16, bf16_caches, None, "NHD")
    assert not pays(16, shape, torch.bfloat16, bf16_caches, None, "NHD")  # cuBLAS + Q/K kernel
    assert not pays(1, shape, torch.float16, bf16_caches, None, "NHD")    # bf16 only
    assert not pays(1, shape, torch.bfloat16, bf16_caches, None, "HND")   # dense NHD only
    fp8 = [torch.zeros(4, 16, 8, 128, dtype=torch.float8_e4m3fn)]
    assert not pays(1, shape, torch.bfloat16, fp8, torch.ones(1), "NHD")  # no fp8 caches
    assert not pays(1, Qwen3AttentionShape(head_dim=64), torch.bfloat16, bf16_caches, None, "NHD")
