"""The sharded path on real GPUs: one process per visible GPU, no collective on
the data path (NCCL only for a barrier). Each rank normalises its own rows and
its own decode sequences (private paged cache, rank-local slots); the parent
process checks the reassembled result against the oracle. Skipped with fewer
than two GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(99)
    rows, hidden = 1000, 4096
    x = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    r = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    tokens, hq, hk = 37, 32, 8
    q = torch.randn(tokens, hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(tokens, hk, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(tokens, hk, 128, generator=g).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    pos = torch.randint(0, 4096, (tokens,), generator=g)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    f = torch.outer(torch.arange(4096, dtype=torch.float32), inv)
    cache = torch.cat((f.cos(), f.sin()), dim=-1)
    return x, r, w, q, k, v, qw, kw, pos, cache


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    import sm120_rmsnorm as ops
    from sm120_rmsnorm.sharding import shard, shard_decode_batch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        x, r, w, q, k, v, qw, kw, pos, cache = _inputs()
        mx, mr = shard(x, world, rank).to(dev), shard(r, world, rank).to(dev)
        ops.fused_add_rms_norm_inplace(mx, mr, w.to(dev))
        lq, lk, lv, lpos = (t.to(dev) for t in shard_decode_batch(world, rank, q, k, v, pos))
        n = lq.shape[0]
        kc = torch.zeros(4, 16, 8, 128, device=dev, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        slots = torch.arange(n, device=dev, dtype=torch.int32)  # rank-local slots
        ops.fused_qk_rms_norm_rope_kv(lq, lk, lv, qw.to(dev), kw.to(dev), lpos, cache.to(dev),
                                      kc, vc, slots)
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])
        torch.save({"x": mx.cpu(), "r": mr.cpu(), "q": lq.cpu(), "k": lk.cpu(),
                    "kc": kc.view(-1, 8, 128)[:n].cpu(), "vc": vc.view(-1, 8, 128)[:n].cpu(),
                    "device": torch.cuda.current_device()},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_all_gpus_shard_rows_and_sequences(tmp_path):
    from gpu_cases import check_norm, check_rope
    from numerics import assert_bitwise_equal
    from oracle import oracle

    oracle.build()
    world = torch.cuda.device_count()
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    parts = [torch.load(tmp_path / f"rank{i}.pt") for i in range(world)]
    assert [p["device"] for p in parts] == list(range(world))
    x, r, w, q, k, v, qw, kw, pos, cache = _inputs()
    want_x, want_r = oracle.fused_add_rms_norm(x, r, w)
    assert_bitwise_equal(torch.cat([p["r"] for p in parts]), want_r, what="residual")
    check_norm(torch.cat([p["x"] for p in parts]), want_x, what="output")
    eq, ek = q.clone(), k.clone()
    oracle.qk_rms_norm_rope_(eq, ek, qw, kw, pos, cache)
    got_q = torch.cat([p["q"] for p in parts])
    got_k = torch.cat([p["k"] for p in parts])
    check_rope(got_q, eq, q, qw, pos, cache, what="query")
    check_rope(got_k, ek, k, kw, pos, cache, what="key")
    assert_bitwise_equal(torch.cat([p["kc"] for p in parts]), got_k, what="key cache")
    assert_bitwise_equal(torch.cat([p["vc"] for p in parts]), v, what="value cache")
