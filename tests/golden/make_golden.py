"""Generate the golden input/output vectors in this directory.

Runs the reference project's own PyTorch oracle (``sm120_rmsnorm/reference.py``,
imported by file path from a checkout of FILWYZ/sm120-norm-fusion-kernels) on
the CPU over seeded inputs, and stores inputs and outputs as ``.npz``. The
fixtures pin the C oracle and, on a GPU, the CUDA kernels. Re-run with

    python tests/golden/make_golden.py --reference /path/to/reference/checkout

bf16 tensors are stored as their raw uint16 bit patterns, with a ``dtype``
entry naming the element type.
"""
from __future__ import annotations

import argparse
import os
import importlib.util
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def load_reference(root: Path):
    spec = importlib.util.spec_from_file_location(
        "reference_oracle", root / "sm120_rmsnorm" / "reference.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def rope_cache(positions: int, theta: float = 1_000_000.0, dim: int = 128) -> torch.Tensor:
    """[positions, dim] fp32 with cos in the first half and sin in the second."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    freqs = torch.outer(torch.arange(positions, dtype=torch.float32), inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def sparse_rope_cache(positions: torch.Tensor, rows: int) -> torch.Tensor:
    """Full-size cache with only the rows that `positions` reads filled in
    (compresses to almost nothing, still exercises large position indices)."""
    dense = rope_cache(int(positions.max()) + 1)
    cache = torch.zeros(rows, 128, dtype=torch.float32)
    cache[positions] = dense[positions]
    return cache


def save(name: str, **arrays) -> None:
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **{k: (to_np(v) if isinstance(v, torch.Tensor) else np.asarray(v))
                                 for k, v in arrays.items()})


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", type=Path, default=None,
                        help="reference checkout (default: $SM120N_REFERENCE_ROOT)")
    args = parser.parse_args()
    if args.reference is None:
        if not os.environ.get("SM120N_REFERENCE_ROOT"):
            parser.error("give --reference or set SM120N_REFERENCE_ROOT")
        args.reference = Path(os.environ["SM120N_REFERENCE_ROOT"])
    ref = load_reference(args.reference)
    eps = 1e-6

    # RMSNorm, the CPU-runnable workload: fp32 x[T, 1024] ~ N(0, 1), w ~ N(1, 0.1).
    for tokens in (1, 4, 16):
        g = torch.Generator().manual_seed(1000 + tokens)
        x = torch.randn(tokens, 1024, generator=g)
        w = 1.0 + 0.1 * torch.randn(1024, generator=g)
        save(f"rms_cpu_t{tokens}", dtype="fp32", x=x, w=w, eps=eps,
             out=ref.rms_norm_reference(x, w, eps))

    # RMSNorm, the reference test shapes (tests/test_correctness.py:19-31).
    for dname, dtype in DTYPES.items():
        for shape in [(1, 1024), (17, 1024), (8, 768), (3, 1000), (2, 4, 2048)]:
            g = torch.Generator().manual_seed(7)
            x = torch.randn(shape, generator=g).to(dtype)
            w = torch.randn(shape[-1], generator=g).to(dtype)
            tag = "x".join(map(str, shape))
            save(f"rms_{dname}_{tag}", dtype=dname, x=x, w=w, eps=eps,
                 out=ref.rms_norm_reference(x, w, eps))

    # Residual add + RMSNorm: reference test shapes (test_correctness.py:34-100)
    # plus B200 widths with w ~ N(1, 0.1).
    fused_cases = [(d, (t, 1024), "randn") for d in DTYPES for t in (1, 7, 24)]
    fused_cases += [("fp16", (5, 768), "randn")]
    fused_cases += [(d, s, "n1") for d in ("bf16", "fp16")
                    for s in [(4, 4096), (16, 2048), (2, 8192), (3, 768)]]
    for dname, shape, wdist in fused_cases:
        dtype = DTYPES[dname]
        g = torch.Generator().manual_seed(11 + shape[0] * 31 + shape[1])
        x = torch.randn(shape, generator=g).to(dtype)
        r = torch.randn(shape, generator=g).to(dtype)
        if wdist == "randn":
            w = torch.randn(shape[-1], generator=g).to(dtype)
        else:
            w = (1.0 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype)
        out, res = ref.fused_add_rms_norm_reference(x, r, w, eps)
        tag = "x".join(map(str, shape))
        save(f"fused_{dname}_{tag}_{wdist}", dtype=dname, x=x, r=r, w=w, eps=eps,
             out=out, res=res)

    # Q/K RMSNorm + RoPE (test_correctness.py:112-138): positions = 3 * arange.
    for dname, dtype in DTYPES.items():
        for tokens in (1, 7):
            for hq, hk in [(16, 8), (4, 2)]:
                g = torch.Generator().manual_seed(29 + tokens + hq)
                q = torch.randn(tokens, hq, 128, generator=g).to(dtype)
                k = torch.randn(tokens, hk, 128, generator=g).to(dtype)
                qw = torch.randn(128, generator=g).to(dtype)
                kw = torch.randn(128, generator=g).to(dtype)
                pos = torch.arange(tokens, dtype=torch.int64) * 3
                cache = rope_cache(tokens * 3 + 1)
                eq, ek = ref.qk_rms_norm_rope_reference(q, k, qw, kw, pos, cache.unsqueeze(1), eps)
                save(f"qk_{dname}_t{tokens}_h{hq}x{hk}", dtype=dname, q=q, k=k, qw=qw, kw=kw,
                     pos=pos, cache=cache, eps=eps, q_out=eq, k_out=ek)

    # Qwen3 batch-1 decode shape: q[1,16,128], k[1,8,128], weights N(1, 0.1),
    # position uniform in [0, 32768) over a 32768-row theta=1e6 cache.
    for dname in ("bf16", "fp16"):
        dtype = DTYPES[dname]
        g = torch.Generator().manual_seed(4242)
        q = torch.randn(1, 16, 128, generator=g).to(dtype)
        k = torch.randn(1, 8, 128, generator=g).to(dtype)
        qw = (1.0 + 0.1 * torch.randn(128, generator=g)).to(dtype)
        kw = (1.0 + 0.1 * torch.randn(128, generator=g)).to(dtype)
        pos = torch.randint(0, 32768, (1,), generator=g, dtype=torch.int64)
        cache = sparse_rope_cache(pos, 32768)
        eq, ek = ref.qk_rms_norm_rope_reference(q, k, qw, kw, pos, cache.unsqueeze(1), eps)
        save(f"qk_decode_{dname}", dtype=dname, q=q, k=k, qw=qw, kw=kw, pos=pos,
             cache=cache, eps=eps, q_out=eq, k_out=ek)

    # Zero input -> zero output (test_correctness.py:141-150).
    for dname in ("bf16", "fp16"):
        dtype = DTYPES[dname]
        q = torch.zeros(2, 16, 128, dtype=dtype)
        k = torch.zeros(2, 8, 128, dtype=dtype)
        w = torch.ones(128, dtype=dtype)
        pos = torch.tensor([0, 511], dtype=torch.int64)
        cache = sparse_rope_cache(pos, 512)
        eq, ek = ref.qk_rms_norm_rope_reference(q, k, w, w, pos, cache.unsqueeze(1), eps)
        save(f"qk_zero_{dname}", dtype=dname, q=q, k=k, qw=w, kw=w, pos=pos, cache=cache,
             eps=eps, q_out=eq, k_out=ek)

    # Q/K + paged KV store (test_correctness.py:163-210): slots = 2 * arange with
    # slots[1] = -1 (padding), random caches so untouched slots are checked too.
    for dname, dtype in DTYPES.items():
        for tokens in (1, 7):
            g = torch.Generator().manual_seed(37 + tokens)
            q = torch.randn(tokens, 16, 128, generator=g).to(dtype)
            k = torch.randn(tokens, 8, 128, generator=g).to(dtype)
            v = torch.randn(tokens, 8, 128, generator=g).to(dtype)
            qw = torch.randn(128, generator=g).to(dtype)
            kw = torch.randn(128, generator=g).to(dtype)
            pos = torch.arange(tokens, dtype=torch.int64) * 2
            cache = rope_cache(tokens * 2 + 1)
            slots = torch.arange(tokens, dtype=torch.int32) * 2
            if tokens > 1:
                slots[1] = -1
            kc = torch.randn(tokens * 2, 8, 128, generator=g).to(dtype)
            vc = torch.randn(tokens * 2, 8, 128, generator=g).to(dtype)
            eq, ek = ref.qk_rms_norm_rope_reference(q, k, qw, kw, pos, cache.unsqueeze(1), eps)
            ekc, evc = kc.clone(), vc.clone()
            valid = slots >= 0
            ekc[slots[valid].long()] = ek[valid]
            evc[slots[valid].long()] = v[valid]
            save(f"qkkv_{dname}_t{tokens}", dtype=dname, q=q, k=k, v=v, qw=qw, kw=kw, pos=pos,
                 cache=cache, slots=slots, kc=kc, vc=vc, eps=eps, q_out=eq, k_out=ek,
                 kc_out=ekc, vc_out=evc)

    total = sum(p.stat().st_size for p in HERE.glob("*.npz"))
    print(f"wrote {len(list(HERE.glob('*.npz')))} fixtures, {total / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
