"""Helpers for GPU parity tests: run the oracle on copies of device tensors."""
from __future__ import annotations

import torch

from numerics import assert_bitwise_equal, assert_rope_close, assert_ulp_close, rope_bound
from oracle import oracle

_ready = False


def _oracle():
    global _ready
    if not _ready:
        oracle.build()
        oracle.set_threads(max(1, min(16, torch.get_num_threads())))
        _ready = True
    return oracle


def cpu(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu").contiguous()


def expect_rms_norm(x, w, eps=1e-6):
    return _oracle().rms_norm(cpu(x), cpu(w), eps)


def expect_fused_add(x, r, w, eps=1e-6):
    return _oracle().fused_add_rms_norm(cpu(x), cpu(r), cpu(w), eps)


def expect_qk(q, k, qw, kw, pos, cache, eps=1e-6):
    q2, k2 = cpu(q).clone(), cpu(k).clone()
    _oracle().qk_rms_norm_rope_(q2, k2, cpu(qw), cpu(kw), cpu(pos), cpu(cache), eps)
    return q2, k2


def expect_qk_kv(q, k, v, qw, kw, pos, cache, kc, vc, slots, eps=1e-6):
    q2, k2, kc2, vc2 = cpu(q).clone(), cpu(k).clone(), cpu(kc).clone(), cpu(vc).clone()
    _oracle().qk_rms_norm_rope_kv_(q2, k2, cpu(v), cpu(qw), cpu(kw), cpu(pos), cpu(cache),
                                   kc2, vc2, cpu(slots), eps)
    return q2, k2, kc2, vc2


def check_norm(actual, expected, what=""):
    assert_ulp_close(actual, expected, what=what)


def check_rope(actual, expected, x_in, w, pos, cache, what=""):
    assert_rope_close(actual, expected, rope_bound(cpu(x_in), cpu(w), cpu(pos), cpu(cache),
                                                   expected), what=what)


__all__ = ["assert_bitwise_equal", "check_norm", "check_rope", "cpu", "expect_fused_add",
           "expect_qk", "expect_qk_kv", "expect_rms_norm"]
