"""bench.py's host-side arithmetic, without a GPU: the repeat summary, the
per-config fractions and strong-scaling efficiency for a sharded
configuration, the row split of the headline, and the DRAM-traffic scaling
from the committed ncu capture."""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


class FakeDist:
    def __init__(self, world, others):
        self.world, self.rank, self.others = world, 0, others

    def max(self, value):
        return max([value, *self.others])


def test_repeat_summary(bench):
    s = bench.repeat_summary([100.0, 102.0, 98.0, 101.0, 99.0], "GB/s")
    assert s["median"] == 100.0 and s["processes"] == 5
    assert s["range_pct"] == pytest.approx(4.0)


def test_per_config_sharded_entry_reports_aggregate_and_efficiency(bench):
    pc = bench.PerConfig.__new__(bench.PerConfig)
    pc.dist, pc.peak, pc.out = FakeDist(2, [10.0]), 1000.0, {}
    # 20 MB in 10 us on the slowest of two ranks; the whole problem alone took 18 us
    e = pc.put("sharded", 8.0, 20_000_000, sharded=True, t1=18.0)
    assert e["us"] == 10.0
    assert e["gbs"] == pytest.approx(2000.0)           # total bytes / max-rank time
    assert e["frac"] == pytest.approx(1.0)             # per GPU: 1000 GB/s of 1000
    assert e["strong_eff"] == pytest.approx(0.9)       # 18 / (2 * 10)
    assert e["sharded"] == "1/2 per GPU"


def test_per_config_replicated_entry_counts_every_rank(bench):
    pc = bench.PerConfig.__new__(bench.PerConfig)
    pc.dist, pc.peak, pc.out = FakeDist(2, [4.0]), 1000.0, {}
    e = pc.put("replicated", 4.0, 1_000_000)
    assert e["gbs"] == pytest.approx(500.0)            # both ranks' bytes
    assert e["frac"] == pytest.approx(0.25)            # per GPU
    assert e["latency_bound"]                          # 1 MB takes 1 us at peak
    assert "strong_eff" not in e


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_headline_rows_are_split_exactly(bench, world):
    bounds = [bench.shard_bounds(bench.HEADLINE_ROWS, world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == bench.HEADLINE_ROWS
    assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) <= 1


def test_traffic_scales_the_committed_capture_by_rows(bench):
    full = bench.dram_traffic_per_launch(65536)
    quarter = bench.dram_traffic_per_launch(16384)
    assert quarter == 1_017_147_136
    assert full == 4 * quarter
    assert full < bench.fused_bytes(65536, 8192, 2)  # no re-reads


def test_byte_models(bench):
    assert bench.fused_bytes(1024, 4096, 2) == 33_562_624
    assert bench.qk_kv_bytes(1024, 32, 8, 2) == 27_800_064
    assert bench.qk_bytes(1, 16, 8, 2) == 1 * (2 * 128 * 48 + 8 + 512) + 512


def test_pytorch_cpu_per_config_names_match_the_gpu_arm(bench):
    """The reference arm's per-configuration CPU timings use the GPU arm's
    per-config names, so the two lines can be read side by side."""
    r = bench.pytorch_cpu_per_config(2)
    expected = {f"rms_norm fp32 {t}x1024" for t in (1, 4, 16, 64, 256)} | \
        {f"qk (no kv) bf16 T={t} 16/8" for t in (1, 4, 16, 64, 256)} | \
        {"fused_add sweep 48 calls (step)", "fused_add bf16 1024x4096 (dominant sweep call)",
         "qk_kv decode bf16 B=1 16/8"}
    assert set(r) == expected
    assert all(v["us"] > 0 and v["gbs"] > 0 for v in r.values())
