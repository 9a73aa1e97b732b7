"""Bounded waits on a kernel's own bulk copies give up safely and are reported.

With the poll limit lowered to one non-blocking poll (sm120n_set_wait_limit),
the row kernels that stage rows in shared memory give up before any copy can
have landed: each block records the expiry in the device fault counter,
waits -- with the full bound -- for its copies to land, and leaves its rows
unwritten. Nothing faults or hangs: every copy is a valid copy that completes
normally; only the wait is shortened. The operator itself stays asynchronous,
so the fault is surfaced by capi.check_device_faults(), which raises. With the
default limit restored, the same calls are correct and record no fault."""
import pytest
import torch

from gpu_cases import assert_bitwise_equal, check_norm, expect_fused_add
from sm120_rmsnorm import capi, fused_add_rms_norm_inplace

pytestmark = pytest.mark.gpu

CASES = [  # rows, hidden: the staged family (auto at 16-128 MiB), the bulk family (24 KiB rows)
    (2048, 4096),
    (64, 12288),
]


def _inputs(rows, hidden, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=g).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(torch.bfloat16)
    return x, r, w


@pytest.mark.parametrize("rows,hidden", CASES)
def test_expired_wait_is_recorded_reported_and_recovers(rows, hidden):
    capi.reset_device_faults()
    x, r, w = _inputs(rows, hidden, rows + hidden)
    capi.set_wait_limit(1)
    try:
        fused_add_rms_norm_inplace(x, r, w)
        torch.cuda.synchronize()
        faults = capi.device_faults()
    finally:
        capi.set_wait_limit(0)
    assert faults > 0, "a one-poll limit must expire before a copy from memory lands"
    with pytest.raises(capi.DeviceFaultError, match="expired"):
        capi.check_device_faults()
    assert capi.device_faults() == 0  # check_device_faults cleared it

    # default limit: the same call is correct and records nothing
    assert capi.wait_limit() == 1 << 22
    x, r, w = _inputs(rows, hidden, rows + hidden + 1)
    expected, expected_res = expect_fused_add(x, r, w)
    fused_add_rms_norm_inplace(x, r, w)
    assert_bitwise_equal(r, expected_res, what="residual")
    check_norm(x.cpu(), expected, what="output")
    capi.check_device_faults()  # does not raise
