"""The N>1 path on CPU: row / sequence sharding across `gloo` ranks.

Each rank normalises only its own rows (the oracle stands in for the GPU
kernel, which needs no collective), the shards are gathered only to check
them, and the result must equal the unsharded computation bit for bit. Also
covered: the max-over-ranks timing aggregation bench.py uses, and a rank that
fails before a collective (the survivor sees an error, nothing hangs).
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sm120_rmsnorm.sharding import shard, shard_bounds, shard_decode_batch


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_rows(mine: torch.Tensor, total: int, world: int) -> torch.Tensor:
    """All ranks' shards in order (padded to the largest shard for gloo, then
    trimmed). Used only to check results."""
    spans = [shard_bounds(total, world, k) for k in range(world)]
    widest = max(b - a for a, b in spans)
    padded = torch.zeros((widest, *mine.shape[1:]), dtype=torch.int32)  # gloo has no int16
    padded[: mine.shape[0]] = mine.to(torch.int32)
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded)
    return torch.cat([p[: b - a] for p, (a, b) in zip(parts, spans)]).to(mine.dtype)


def _init(rank, world, port, timeout_s=30):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_bounds_partition_every_size(world):
    for total in range(0, 70):
        spans = [shard_bounds(total, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == total
        for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
            assert a1 == b0
        sizes = [b - a for a, b in spans]
        assert max(sizes) - min(sizes) <= 1


def test_shard_rejects_bad_ranks():
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)
    with pytest.raises(ValueError):
        shard_decode_batch(2, 0, torch.zeros(3), torch.zeros(4))


def _fused_worker(rank, world, port, rows, hidden, result_path):
    from oracle import oracle
    _init(rank, world, port)
    try:
        g = torch.Generator().manual_seed(2024)
        x = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
        r = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
        mine_x, mine_r = shard(x, world, rank).clone(), shard(r, world, rank).clone()
        oracle.set_threads(1)
        oracle.fused_add_rms_norm_out(mine_x, mine_r, w, mine_x, mine_r)
        # gather the shards (check only; the operator itself never communicates)
        whole = _gather_rows(mine_x.view(torch.int16), rows, world).view(torch.bfloat16)
        if rank == 0:
            oracle.set_threads(2)
            full_x, full_r = x.clone(), r.clone()
            oracle.fused_add_rms_norm_out(full_x, full_r, w, full_x, full_r)
            torch.save({"equal": torch.equal(whole.view(torch.int16), full_x.view(torch.int16))},
                       result_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows", [7, 64])
def test_two_rank_sharded_rows_equal_the_unsharded_result(tmp_path, rows):
    from oracle import oracle
    oracle.build()
    out = tmp_path / "result.pt"
    mp.spawn(_fused_worker, args=(2, _free_port(), rows, 1024, str(out)), nprocs=2, join=True)
    assert torch.load(out)["equal"]


def _decode_worker(rank, world, port, result_path):
    from oracle import oracle
    _init(rank, world, port)
    try:
        tokens, hq, hk = 9, 4, 2
        g = torch.Generator().manual_seed(5)
        q = torch.randn(tokens, hq, 128, generator=g).to(torch.bfloat16)
        k = torch.randn(tokens, hk, 128, generator=g).to(torch.bfloat16)
        v = torch.randn(tokens, hk, 128, generator=g).to(torch.bfloat16)
        w = torch.ones(128, dtype=torch.bfloat16)
        cache = torch.randn(64, 128, generator=g)
        pos = torch.randint(0, 64, (tokens,), generator=g)
        # each rank owns a private paged cache: rank-local slots 0..n-1
        lq, lk, lv, lpos = (t.clone() for t in shard_decode_batch(world, rank, q, k, v, pos))
        n = lq.shape[0]
        kc = torch.zeros(16, hk, 128, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        oracle.qk_rms_norm_rope_kv_(lq, lk, lv, w, w, lpos, cache, kc, vc,
                                    torch.arange(n, dtype=torch.int32))
        gathered = _gather_rows(kc[:n].view(torch.int16).contiguous(), tokens, world)
        if rank == 0:
            fq, fk = q.clone(), k.clone()
            oracle.qk_rms_norm_rope_(fq, fk, w, w, pos, cache)
            torch.save({"equal": torch.equal(gathered, fk.view(torch.int16))}, result_path)
    finally:
        dist.destroy_process_group()


def test_two_rank_decode_sequences_with_private_caches(tmp_path):
    from oracle import oracle
    oracle.build()
    out = tmp_path / "result.pt"
    mp.spawn(_decode_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    assert torch.load(out)["equal"]


def _max_worker(rank, world, port, result_path):
    _init(rank, world, port)
    try:
        t = torch.tensor([1.5 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            torch.save({"max": float(t)}, result_path)
    finally:
        dist.destroy_process_group()


def test_two_rank_time_is_the_maximum_over_ranks(tmp_path):
    out = tmp_path / "result.pt"
    mp.spawn(_max_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    assert torch.load(out)["max"] == 2.5


def _failing_worker(rank, world, port):
    _init(rank, world, port, timeout_s=5)
    try:
        if rank == 1:
            raise RuntimeError("rank 1 failed before its collective")
        dist.barrier()  # rank 0 waits for a peer that is gone
    finally:
        dist.destroy_process_group()


def test_a_failed_rank_surfaces_as_an_error():
    with pytest.raises(Exception) as err:
        mp.spawn(_failing_worker, args=(2, _free_port()), nprocs=2, join=True)
    assert "rank 1 failed" in str(err.value) or "terminated" in str(err.value).lower()
