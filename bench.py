"""Benchmark: achieved HBM GB/s (% of B200 peak) and us/call of the fused
normalisation path, at 1..8 GPUs.

Headline workload (one "step"): the in-place residual-add + RMSNorm prefill,
bf16 x and residual [65536, 8192] ~ N(0, 1), weight [8192] ~ N(1, 0.1), eps
1e-6 -- one call of ``fused_add_rms_norm_inplace`` per step on each GPU's
share of the rows. Under torchrun the 65536 rows are split evenly across the
ranks (``sharding.shard_bounds``), so the total problem is fixed as N grows
(strong scaling) and no collective touches the data path. ``value`` = the
algorithmic bytes of the whole problem / the max-over-ranks device time per
step. Each rank's x + residual (2 GiB / N, >= 268 MB at N = 8) is larger than
L2 (126 MB), so steps run back to back without an L2 flush.

Also on the line:
  * ``roofline`` -- the headline kernel (one launch per step): algorithmic
    bytes per launch over its launch duration, against the measured HBM copy
    peak; its ``per_config`` table covers every workload configuration
    (us/call, GB/s, fraction of peak, strong-scaling data for the sharded
    ones, and comparators at N = 1), and ``repeat`` the headline measured in
    5 independent processes x 3 samples (N = 1);
  * ``e2e`` -- the headline through the public API with x and residual
    uploaded from pinned host memory and both results downloaded, every step,
    inside the timed region;
  * ``cpu_baseline`` -- the C restatement of the reference's CPU path on the
    host cores (rank 0, N = 1 only), on a bounded sample of the workload.

Per-config timing: a CUDA graph of R back-to-back calls on R distinct buffer
sets (R <= 64, at most 256 MiB in all, so every call reads data that is not
in L2), replayed after an L2 flush (a 512 MiB write, outside the timed
events); us/call = replay time / R.

``--impl reference`` times the reference path's CPU implementation (the C
restatement of its PyTorch oracle, all host threads) on the headline workload
in 5 independent processes, and the reference's own CUDA kernels on the same
workload on this GPU. ``--detail FILE`` also runs the engine-side extension,
engine and projection suites and writes them to FILE.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "sm120-norm-fusion-kernels_b200"))
sys.path.insert(0, str(ROOT))

TOKENS = (1, 4, 16, 64, 256, 1024)
HIDDEN = (768, 1024, 2048, 4096)
DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16}
EPS = 1e-6
FLUSH_BYTES = 512 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
HEADLINE_ROWS, HEADLINE_HIDDEN = 65536, 8192
HEADLINE_WORKLOAD = ("in-place residual add + RMSNorm prefill, bf16 x and residual "
                     "[65536, 8192] ~ N(0,1), weight ~ N(1,0.1), eps 1e-6; rows split evenly "
                     "across the GPUs")
METRIC = "achieved HBM GB/s (% of B200 peak) and us/call per op at 1/2/4/8 GPUs"
REPEAT_PROCESSES, REPEAT_SAMPLES = 5, 3


# ---------------------------------------------------------------------------
# byte models (algorithmic bytes per call)
# ---------------------------------------------------------------------------
def fused_bytes(t: int, h: int, s: int) -> int:
    return 4 * t * h * s + h * s  # read x, r; write x, r; weight once


def rms_bytes(t: int, h: int, s: int) -> int:
    return 2 * t * h * s + h * s


def qk_kv_bytes(t: int, hq: int, hk: int, s: int, d: int = 128) -> int:
    # q, k read + written; v read; k-cache and v-cache written; position (8 B),
    # slot (4 B) and one fp32 cos/sin row (4 * d B) per token; two weights once.
    return t * (s * d * (2 * hq + 5 * hk) + 8 + 4 + 4 * d) + 2 * d * s


def qk_bytes(t: int, hq: int, hk: int, s: int, d: int = 128) -> int:
    # q, k read + written; position and one cos/sin row per token; weights once
    return t * (s * d * (2 * hq + 2 * hk) + 8 + 4 * d) + 2 * d * s


def sweep_shapes():
    return [(t, h, name) for name in DTYPES for t in TOKENS for h in HIDDEN]


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    from sm120_rmsnorm.sharding import shard_bounds as bounds
    return bounds(total, world, rank)


# ---------------------------------------------------------------------------
# environment
# ---------------------------------------------------------------------------
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self):
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            torch.cuda.set_device(self.local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device("cuda", self.local_rank))
            self.pg = dist
        else:
            torch.cuda.set_device(0)

    def barrier(self):
        torch.cuda.synchronize()
        if self.pg is not None:
            self.pg.barrier(device_ids=[self.local_rank])
        torch.cuda.synchronize()

    def max(self, value: float) -> float:
        if self.pg is None:
            return value
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def measured_hbm_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy burst)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s pool figure; MEASURED_PEAKS.json absent)"


def dram_traffic_per_launch(rows: int):
    """DRAM bytes read + written by one launch of the headline kernel on `rows`
    rows, scaled by rows from the committed ncu capture of a smaller launch of
    the same kernel (profiles/dram_traffic.txt), or None."""
    path = ROOT / "profiles" / "dram_traffic.txt"
    if not path.exists():
        return None
    out = {}
    for line in path.read_text().splitlines():
        if "=" in line and not line.startswith("#"):
            k, v = line.split("=", 1)
            out[k.strip()] = v.strip()
    try:
        captured_rows = int(out["rows"])
        per_launch = float(out["dram_bytes_per_launch"])
    except (KeyError, ValueError):
        return None
    if out.get("hidden") != str(HEADLINE_HIDDEN):
        return None
    return int(per_launch * rows / captured_rows)


def sampled_gpus(world: int) -> str:
    """nvidia-smi ids of the GPUs this job runs on."""
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        return ",".join(v.strip() for v in visible.split(",")[:world])
    return ",".join(str(i) for i in range(world))


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: str | None):
        self.gpus = gpus
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        if self.gpus is None:
            return self
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
               "-lms", "100"]
        if self.gpus:
            cmd += ["-i", self.gpus]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)

    def summary(self):
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((int(parts[0]), float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, flag in enumerate(r[3])
                          if flag.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in rows),
                "sm_max_mhz": max(r[2] for r in rows), "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------
class Flusher:
    def __init__(self):
        self.buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def __call__(self):
        self.buf.fill_(1)


def event_pair():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def capture(fns):
    """A CUDA graph of the calls in `fns` (each run once first, so lazy kernel
    loading and compilation stay out of it)."""
    for fn in fns:
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for fn in fns:
            fn()
    return graph, []


def time_graph(graph, flush: "Flusher", reps: int) -> float:
    """Mean device time (us) of one replay, L2 flushed before every replay
    (outside the timed events)."""
    total = 0.0
    for _ in range(reps):
        flush()
        a, b = event_pair()
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        total += a.elapsed_time(b) * 1e3
    return total / reps


def time_calls(calls, flush: "Flusher", reps: int, eager_fallback: bool = False
               ) -> tuple[float, str]:
    """us per call of `calls` (R calls on R distinct buffer sets) by the graph
    protocol. With `eager_fallback` (library comparators only), calls that
    cannot be captured in a CUDA graph are timed as an eager back-to-back loop
    after the same flush; this package's own calls always capture, and a
    failure there propagates."""
    try:
        graph, _ = capture(calls)
    except Exception:  # noqa: BLE001 - re-raised unless this is a comparator
        if not eager_fallback:
            raise
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(reps):
            flush()
            a, b = event_pair()
            a.record()
            for fn in calls:
                fn()
            b.record()
            b.synchronize()
            total += a.elapsed_time(b) * 1e3
        return total / reps / len(calls), "eager loop"
    us = time_graph(graph, flush, reps) / len(calls)
    del graph
    return us, "graph"


def sets_for(nbytes: int) -> int:
    """Distinct buffer sets per timed graph: up to 64, at most 256 MiB in all."""
    return max(1, min(64, (256 << 20) // max(nbytes, 1)))


def sm_copy_calls(nbytes: int, g: torch.Generator) -> list:
    """Calls of a plain elementwise kernel on the SMs (d = s * 1, bf16) that
    reads nbytes / 2 and writes nbytes / 2, on distinct buffer sets: the
    protocol's own floor for a call that moves nbytes (a same-dtype copy_ in a
    graph runs on the copy engines instead)."""
    n = max(1, nbytes // 4)
    pairs = [(torch.randn(n, device="cuda", generator=g).to(torch.bfloat16),
              torch.empty(n, device="cuda", dtype=torch.bfloat16))
             for _ in range(sets_for(nbytes))]
    return [lambda s=s, d=d: torch.mul(s, 1, out=d) for s, d in pairs]


def rope_table(n: int, rotary: int = 128, device="cuda", dtype=torch.float32):
    inv = 1.0 / (1e6 ** (torch.arange(0, rotary, 2, dtype=torch.float32, device=device) / rotary))
    f = torch.outer(torch.arange(n, dtype=torch.float32, device=device), inv)
    return torch.cat((f.cos(), f.sin()), dim=-1).to(dtype)


# ---------------------------------------------------------------------------
# headline: the prefill residual add + RMSNorm, rows sharded over the ranks
# ---------------------------------------------------------------------------
class PrefillRows:
    """This rank's rows of the headline workload on its GPU."""

    def __init__(self, rows: int, seed: int, device="cuda"):
        g = torch.Generator(device=device).manual_seed(seed)
        h = HEADLINE_HIDDEN
        self.rows = rows
        self.x = torch.randn(rows, h, device=device, generator=g).to(torch.bfloat16)
        self.r = torch.randn(rows, h, device=device, generator=g).to(torch.bfloat16)
        self.w = (1 + 0.1 * torch.randn(h, device=device, generator=g)).to(torch.bfloat16)
        self.bytes = fused_bytes(rows, h, 2)

    def call(self, ops):
        ops.fused_add_rms_norm_inplace(self.x, self.r, self.w, EPS)


def headline_step_ms(ops, head: PrefillRows, steps: int, warmup: int, dist: "Dist") -> float:
    """Device time per step (one call on this rank's rows), CUDA events around
    exactly `steps` back-to-back calls, barrier + synchronize on both sides."""
    for _ in range(warmup):
        head.call(ops)
    dist.barrier()
    a, b = event_pair()
    a.record()
    for _ in range(steps):
        head.call(ops)
    b.record()
    dist.barrier()
    return a.elapsed_time(b) / steps


def e2e_headline(ops, head: PrefillRows, steps: int, dist: "Dist") -> dict:
    """The headline through sm120_rmsnorm.fused_add_rms_norm_inplace with host
    buffers: every step uploads this rank's x and residual (one packed pinned
    buffer, one copy), runs the call on views of the device copy and downloads
    both results (one copy). Three device buffer sets rotate over three
    streams, so a step's upload overlaps the previous step's call and
    download; per-step time = elapsed / steps (max over ranks)."""
    n = head.x.numel() * head.x.element_size()
    total = 2 * n
    host_in = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    host_out = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    host_in[:n].view(torch.bfloat16).copy_(head.x.view(-1))
    host_in[n:].view(torch.bfloat16).copy_(head.r.view(-1))
    dev_sets = [torch.empty(total, dtype=torch.uint8, device="cuda") for _ in range(3)]
    shape = (head.rows, HEADLINE_HIDDEN)
    views = [(b[:n].view(torch.bfloat16).view(shape), b[n:].view(torch.bfloat16).view(shape))
             for b in dev_sets]
    up, compute, down = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()

    def run(n_steps):
        origin = torch.cuda.current_stream()
        for stream in (up, compute, down):
            stream.wait_stream(origin)
        freed = [None] * len(dev_sets)
        for k in range(n_steps):
            i = k % len(dev_sets)
            with torch.cuda.stream(up):
                if freed[i] is not None:
                    up.wait_event(freed[i])
                dev_sets[i].copy_(host_in, non_blocking=True)
                uploaded = torch.cuda.Event()
                uploaded.record(up)
            compute.wait_event(uploaded)
            with torch.cuda.stream(compute):
                x, r = views[i]
                ops.fused_add_rms_norm_inplace(x, r, head.w, EPS)
                computed = torch.cuda.Event()
                computed.record(compute)
            down.wait_event(computed)
            with torch.cuda.stream(down):
                host_out.copy_(dev_sets[i], non_blocking=True)
                freed[i] = torch.cuda.Event()
                freed[i].record(down)
        for stream in (up, compute, down):
            origin.wait_stream(stream)

    run(2)  # warm-up
    e2e_steps = max(6, steps // 2)
    dist.barrier()
    a, b = event_pair()
    a.record()
    run(e2e_steps)
    b.record()
    dist.barrier()
    ms = dist.max(a.elapsed_time(b) / e2e_steps)
    del dev_sets, views, host_in, host_out
    torch.cuda.empty_cache()
    return {"value": round(fused_bytes(HEADLINE_ROWS, HEADLINE_HIDDEN, 2) / (ms * 1e-3) / 1e9, 2),
            "unit": "GB/s", "ms_per_step": round(ms, 3),
            "h2d_bytes_per_step": total * dist.world, "d2h_bytes_per_step": total * dist.world,
            "path": "sm120_rmsnorm.fused_add_rms_norm_inplace on views of one packed device "
                    "buffer per step and rank: one pinned-host upload of x and residual and one "
                    "download of both results per step, three device buffer sets rotating over "
                    f"three streams, {e2e_steps} steps timed"}


# ---------------------------------------------------------------------------
# comparators (N = 1 only; never on the product path)
# ---------------------------------------------------------------------------
class ReferenceKernels:
    """The reference project's own CUDA kernels (compiled for sm_100a from its
    sources by oracle/build_ref.py), called with its ops.py default versions."""

    def __init__(self, module):
        self.m = module

    @classmethod
    def load(cls):
        from oracle import build_ref
        module = build_ref.load()
        return None if module is None else cls(module)

    def fused_add_rms_norm_inplace(self, x, r, w, eps=EPS, version=0):
        self.m.fused_add_rms_norm_inplace(x, r, w, eps, version)

    def rms_norm_out(self, x, w, out, eps=EPS, version=2):
        self.m.rms_norm_out(x, w, out, eps, version)

    def fused_qk_rms_norm_rope(self, q, k, qw, kw, pos, cache, eps=EPS, version=2):
        self.m.fused_qk_rms_norm_rope(q, k, qw, kw, pos, cache, eps, version)

    def fused_qk_rms_norm_rope_kv(self, q, k, v, qw, kw, pos, cache, kc, vc, slots, eps=EPS,
                                  version=1):
        self.m.fused_qk_rms_norm_rope_kv(q, k, v, qw, kw, pos, cache, kc, vc, slots, eps, version)


def vllm_ops():
    """torch.ops._C / _C_cache_ops from the installed vLLM build, as an
    industrial comparator (never on the product path), or None."""
    try:
        import importlib.util
        spec = importlib.util.find_spec("vllm")
        if spec is None or not spec.submodule_search_locations:
            return None
        root = Path(list(spec.submodule_search_locations)[0])
        for name in ("_C.abi3.so", "_C_stable_libtorch.abi3.so"):  # both register ops
            torch.ops.load_library(str(root / name))
        return torch.ops._C, torch.ops._C_cache_ops
    except Exception:  # noqa: BLE001 - a missing comparator is reported, not fatal
        return None


def flashinfer_fused_add_rmsnorm():
    """FlashInfer's in-place residual add + RMSNorm (an installed library
    kernel, timed as a comparator only), or None when it does not load."""
    try:
        from flashinfer import norm
        return norm.fused_add_rmsnorm
    except Exception:  # noqa: BLE001 - optional comparator
        return None


def torch_native_fused(x, r, w):
    """The reference benchmark's PyTorch-native arm: ``x + r`` then
    ``F.rms_norm`` (out of place, two kernels)."""
    import torch.nn.functional as F
    summed = x + r
    return F.rms_norm(summed, (x.shape[-1],), w, EPS), summed


_COMPILED = {}


def compiled(fn):
    """torch.compile of a comparator function (fullgraph, static shapes), once
    per function."""
    if fn not in _COMPILED:
        _COMPILED[fn] = torch.compile(fn, fullgraph=True, dynamic=False)
    return _COMPILED[fn]


def qk_reference_math(q, k, qw, kw, pos, cache):
    from sm120_rmsnorm.reference import qk_rms_norm_rope_reference
    return qk_rms_norm_rope_reference(q, k, qw, kw, pos, cache, EPS)


# ---------------------------------------------------------------------------
# per-config table
# ---------------------------------------------------------------------------
class PerConfig:
    """us/call, GB/s and fraction of the HBM peak for every workload
    configuration, timed by the graph protocol (module docstring). Sharded
    configurations give each rank its share of the tokens / rows (own KV cache,
    rank-local slots); at N > 1 rank 0 also times the whole problem alone
    (``t1_us``) so the line carries strong-scaling efficiency
    t1 / (N * tN). Comparators run at N = 1 only."""

    def __init__(self, ops, flush, dist, args, peak):
        self.ops, self.flush, self.dist, self.args, self.peak = ops, flush, dist, args, peak
        self.reps = max(3, args.reps)
        self.out = {}
        self.g = torch.Generator(device="cuda").manual_seed(99 + dist.rank)
        self.cpu_g = torch.Generator().manual_seed(7 + dist.rank)
        want_cmp = dist.world == 1 and not args.skip_comparators
        self.cmp_on = want_cmp
        self.ref = ReferenceKernels.load() if want_cmp else None
        self.cache = rope_table(32768)

    # -- helpers ---------------------------------------------------------------
    def us(self, calls) -> float:
        us, _ = time_calls(calls, self.flush, self.reps)
        return us

    def comparators(self, build: dict) -> dict:
        """{name: us} for each comparator builder (name -> () -> calls);
        failures are recorded as unavailable."""
        out = {}
        if not self.cmp_on:
            return out
        for name, make in build.items():
            if make is None:
                continue
            try:
                calls = make()
                us, how = time_calls(calls, self.flush, self.reps, eager_fallback=True)
                out[name] = round(us, 2) if how == "graph" else [round(us, 2), how]
                del calls
            except Exception as e:  # noqa: BLE001 - comparators may be unavailable
                out[name] = f"unavailable: {type(e).__name__}: {str(e)[:80]}"
                torch.cuda.synchronize()
        return out

    def put(self, name, us_local, nbytes, sharded=False, t1=None, cmp=None, latency_floor=2.0):
        d = self.dist
        us = d.max(us_local)
        gbs = nbytes / (us * 1e-6) / 1e9
        per_gpu = gbs / (d.world if sharded else 1)
        if not sharded:
            gbs *= d.world  # replicated: every rank moves nbytes
        e = {"us": round(us, 3), "gbs": round(gbs, 1), "frac": round(per_gpu / self.peak, 3)}
        if nbytes / (self.peak * 1e3) < latency_floor:  # bytes take < ~2 us at peak
            e["latency_bound"] = True
        if sharded and d.world > 1:
            e["sharded"] = f"1/{d.world} per GPU"
            if t1 is not None:
                e["t1_us"] = round(t1, 3)
                e["strong_eff"] = round(t1 / (d.world * us), 3)
        if cmp:
            e["cmp_us"] = cmp
        self.out[name] = e
        return e

    def whole_on_rank0(self, build) -> float | None:
        """Rank 0 times the unsharded problem alone (others wait); None at N = 1."""
        d = self.dist
        if d.world == 1:
            return None
        d.barrier()
        us = 0.0
        if d.rank == 0:
            calls = build(0, None)
            us = self.us(calls)
            del calls
            torch.cuda.empty_cache()
        d.barrier()
        return d.max(us)

    # -- configurations ----------------------------------------------------------
    def rms_fp32(self):
        """fp32 RMSNorm rows of 1024 (the reference's CPU-runnable workload)."""
        g = self.g
        for t in (1, 4, 16, 64, 256):
            nbytes = rms_bytes(t, 1024, 4)
            sets = []
            for _ in range(sets_for(nbytes)):
                x = torch.randn(t, 1024, device="cuda", generator=g)
                w = 1.0 + 0.1 * torch.randn(1024, device="cuda", generator=g)
                sets.append((x, w, torch.empty_like(x)))
            calls = [lambda s=s: self.ops.rms_norm_out(s[0], s[1], s[2], EPS) for s in sets]
            cmp = self.comparators({
                "reference_kernels": self.ref and (lambda: [
                    lambda s=s: self.ref.rms_norm_out(s[0], s[1], s[2], EPS, 2) for s in sets])})
            self.put(f"rms_norm fp32 {t}x1024", self.us(calls), nbytes, cmp=cmp)

    def sweep(self):
        """The fused add + RMSNorm sweep: step time of the 48 calls as one graph
        and each shape's per-call time (replicated on every rank)."""
        g = self.g
        items = []
        for t, h, name in sweep_shapes():
            dt = DTYPES[name]
            x = torch.randn(t, h, device="cuda", generator=g).to(dt)
            r = torch.randn(t, h, device="cuda", generator=g).to(dt)
            w = (1.0 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(dt)
            items.append((t, h, name, x, r, w))
        step_bytes = sum(fused_bytes(t, h, 2) for t, h, *_ in items)

        def step(ops):
            return [lambda: [ops.fused_add_rms_norm_inplace(x, r, w, EPS)
                             for *_, x, r, w in items]]

        step_us = self.us(step(self.ops))
        cmp = self.comparators({"reference_kernels": self.ref and (lambda: step(self.ref))})
        e = self.put("fused_add sweep 48 calls (step)", step_us, step_bytes, cmp=cmp)
        shapes = {}
        for t, h, name, x, r, w in items:
            nbytes = fused_bytes(t, h, 2)
            bufs = [(x, r)] + [(torch.randn(t, h, device="cuda", generator=g).to(x.dtype),
                                torch.randn(t, h, device="cuda", generator=g).to(x.dtype))
                               for _ in range(sets_for(nbytes) - 1)]
            us = self.dist.max(self.us([lambda bx=bx, br=br, w=w: self.ops.fused_add_rms_norm_inplace(
                bx, br, w, EPS) for bx, br in bufs]))
            shapes[f"{name} {t}x{h}"] = [round(us, 2), round(nbytes / (us * 1e-6) / 1e9, 1)]
            del bufs
        e["per_shape_us_gbs"] = shapes
        return items

    def fused_add_comparators(self, t, h):
        """The headline op at one shape beside the reference's kernels, PyTorch
        native (x + r; F.rms_norm), its torch.compile, FlashInfer and vLLM."""
        g = self.g
        nbytes = fused_bytes(t, h, 2)
        w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(torch.bfloat16)
        sets = [(torch.randn(t, h, device="cuda", generator=g).to(torch.bfloat16),
                 torch.randn(t, h, device="cuda", generator=g).to(torch.bfloat16))
                for _ in range(sets_for(nbytes))]
        ours = self.us([lambda x=x, r=r: self.ops.fused_add_rms_norm_inplace(x, r, w, EPS)
                        for x, r in sets])
        vllm = vllm_ops()
        fi = flashinfer_fused_add_rmsnorm()
        native_c = compiled(torch_native_fused)
        # out-of-place comparators keep every call's outputs alive, so each call
        # writes its own fresh buffers (a freed output would be reused by the next
        # call and its writes would stay in L2)
        keep = [None] * len(sets)

        def kept(fn):
            return [lambda i=i, x=x, r=r: keep.__setitem__(i, fn(x, r, w))
                    for i, (x, r) in enumerate(sets)]

        cmp = self.comparators({
            "sm_copy_same_bytes": lambda: sm_copy_calls(nbytes, g),
            "reference_kernels": self.ref and (lambda: [
                lambda x=x, r=r: self.ref.fused_add_rms_norm_inplace(x, r, w) for x, r in sets]),
            "torch_native": lambda: kept(torch_native_fused),
            "torch_compile": lambda: kept(native_c),
            "flashinfer": fi and (lambda: [lambda x=x, r=r: fi(x, r, w, EPS) for x, r in sets]),
            "vllm": vllm and (lambda: [lambda x=x, r=r: vllm[0].fused_add_rms_norm(x, r, w, EPS)
                                       for x, r in sets]),
        })
        del sets, keep
        return ours, nbytes, cmp

    def qk_kv(self, name, b_total, hq, hk, blocks, contiguous, sharded):
        """Q/K norm + RoPE + paged KV store; sharded over sequences (tokens)."""
        d = self.dist

        def build(start, stop, ops=None):
            ops = ops or self.ops
            if stop is None:
                start, stop = 0, b_total
            b = stop - start
            nbytes = qk_kv_bytes(b, hq, hk, 2)
            n_sets = sets_for(nbytes)
            bf = torch.bfloat16
            kc = torch.zeros(blocks, 16, hk, 128, device="cuda", dtype=bf)
            vc = torch.zeros_like(kc)
            qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=self.g)).to(bf)
            kw = (1 + 0.1 * torch.randn(128, device="cuda", generator=self.g)).to(bf)
            all_slots = torch.randperm(blocks * 16, generator=self.cpu_g)[: b * n_sets]
            calls = []
            for i in range(n_sets):
                q = torch.randn(b, hq, 128, device="cuda", generator=self.g).to(bf)
                k = torch.randn(b, hk, 128, device="cuda", generator=self.g).to(bf)
                v = torch.randn(b, hk, 128, device="cuda", generator=self.g).to(bf)
                if contiguous:  # prefill: positions of this shard, rank-local contiguous slots
                    pos = torch.arange(start, stop, device="cuda")
                    slots = torch.arange(b, device="cuda", dtype=torch.int32)
                else:  # decode: distinct random positions, unique random slots
                    pos = torch.randperm(32768, generator=self.cpu_g)[:b].cuda()
                    slots = all_slots[i * b:(i + 1) * b].to(torch.int32).cuda()
                calls.append(lambda q=q, k=k, v=v, pos=pos, slots=slots:
                             ops.fused_qk_rms_norm_rope_kv(q, k, v, qw, kw, pos, self.cache, kc,
                                                           vc, slots, EPS))
            return calls

        if sharded:
            start, stop = shard_bounds(b_total, d.world, d.rank)
        else:
            start, stop = 0, b_total
        calls = build(start, stop)
        us = self.us(calls)
        del calls
        torch.cuda.empty_cache()
        t1 = self.whole_on_rank0(lambda s, e: build(s, e)) if sharded else None
        nbytes = qk_kv_bytes(b_total, hq, hk, 2)
        cmp = self.comparators({
            "sm_copy_same_bytes": lambda: sm_copy_calls(nbytes, self.g),
            "reference_kernels": self.ref and (lambda: build(0, b_total, self.ref))})
        torch.cuda.empty_cache()
        return self.put(name, us, nbytes, sharded=sharded, t1=t1, cmp=cmp)

    def qk_no_kv(self):
        """Q/K norm + RoPE without the KV store (16 / 8 heads, positions
        0..T-1), beside the reference's kernel and the eager / compiled
        PyTorch statement of the math, as the reference's own benchmark
        times it."""
        bf = torch.bfloat16
        compiled_math = compiled(qk_reference_math)
        for t in (1, 4, 16, 64, 256):
            nbytes = qk_bytes(t, 16, 8, 2)
            qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=self.g)).to(bf)
            kw = (1 + 0.1 * torch.randn(128, device="cuda", generator=self.g)).to(bf)
            pos = torch.arange(t, device="cuda")
            sets = [(torch.randn(t, 16, 128, device="cuda", generator=self.g).to(bf),
                     torch.randn(t, 8, 128, device="cuda", generator=self.g).to(bf))
                    for _ in range(sets_for(nbytes))]
            us = self.us([lambda q=q, k=k: self.ops.fused_qk_rms_norm_rope(
                q, k, qw, kw, pos, self.cache, EPS) for q, k in sets])
            keep = [None] * len(sets)  # every call's outputs stay alive (fresh buffers)

            def kept(fn):
                return [lambda i=i, q=q, k=k: keep.__setitem__(i, fn(q, k, qw, kw, pos, self.cache))
                        for i, (q, k) in enumerate(sets)]

            cmp = self.comparators({
                "reference_kernels": self.ref and (lambda: [
                    lambda q=q, k=k: self.ref.fused_qk_rms_norm_rope(q, k, qw, kw, pos, self.cache)
                    for q, k in sets]),
                "torch_eager": lambda: kept(qk_reference_math),
                "torch_compile": lambda: kept(compiled_math),
            })
            self.put(f"qk (no kv) bf16 T={t} 16/8", us, nbytes, cmp=cmp)
            del sets, keep

    def engine_formats(self):
        """The engine-side extensions at their prefill / decode sizes beside
        vLLM's kernels doing the same work (N = 1 only): the generalised Q/K
        norm + RoPE + cache store on strided QKV views (bf16 and fp8 NHD
        caches), and residual add + RMSNorm with fp8 and NVFP4 outputs."""
        from sm120_rmsnorm import extensions as ext

        bf = torch.bfloat16
        g, cpu_g = self.g, self.cpu_g
        vllm = vllm_ops()
        one = torch.ones(1, device="cuda")
        qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
        kw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
        cache_bf = self.cache.to(bf)
        for name, b, hq, hk, blocks, fp8, contiguous in (
                ("ext qk_cache prefill 32768 tok 64/8 strided qkv, bf16 NHD cache",
                 32768, 64, 8, 2048, False, True),
                ("ext qk_cache decode B=1024 32/8 strided qkv, fp8 NHD cache",
                 1024, 32, 8, 65536, True, False)):
            nbytes = qk_cache_bytes(b, hq, hk, 2, cache_elem=1 if fp8 else 2)
            kc = torch.zeros(blocks, 16, hk, 128, device="cuda",
                             dtype=torch.float8_e4m3fn if fp8 else bf)
            vc = torch.zeros_like(kc)
            sets = []
            all_slots = torch.randperm(blocks * 16, generator=cpu_g)
            for i in range(sets_for(nbytes)):
                qkv = torch.randn(b, (hq + 2 * hk) * 128, device="cuda", generator=g).to(bf)
                if contiguous:
                    pos = torch.arange(b, device="cuda")
                    slots = torch.arange(b, device="cuda", dtype=torch.int32)
                else:
                    pos = torch.randperm(32768, generator=cpu_g)[:b].cuda()
                    slots = all_slots[i * b:(i + 1) * b].to(torch.int32).cuda()
                sets.append((qkv, qkv[:, :hq * 128].view(b, hq, 128),
                             qkv[:, hq * 128:(hq + hk) * 128].view(b, hk, 128),
                             qkv[:, (hq + hk) * 128:].view(b, hk, 128), pos, slots))
            scales = (one, one) if fp8 else (None, None)
            us = self.us([lambda s=s: ext.qk_norm_rope_cache_(
                s[1], s[2], s[3], qw, kw, s[4], self.cache, kc, vc, s[5], *scales)
                for s in sets])
            cmp = {}
            if vllm is not None:
                C, cache_ops = vllm
                vkc = torch.zeros(blocks, 16, hk, 128, device="cuda",
                                  dtype=torch.uint8 if fp8 else bf)
                vvc = torch.zeros_like(vkc)
                kind = "fp8" if fp8 else "auto"

                def unfused(s):
                    C.fused_qk_norm_rope(s[0], hq, hk, hk, 128, EPS, qw, kw, cache_bf, True, s[4])
                    cache_ops.reshape_and_cache_flash(s[2], s[3], vkc, vvc, s[5].long(), kind,
                                                      one, one)

                cmp = self.comparators({"vllm_qk_norm_rope_and_reshape_and_cache":
                                        lambda: [lambda s=s: unfused(s) for s in sets]})
                del vkc, vvc
            self.put(name, us, nbytes, cmp=cmp)
            del sets, kc, vc
            torch.cuda.empty_cache()

        t, h = HEADLINE_ROWS, HEADLINE_HIDDEN
        w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(bf)
        x = torch.randn(t, h, device="cuda", generator=g).to(bf)
        r = torch.randn(t, h, device="cuda", generator=g).to(bf)
        scale = torch.full((1,), 0.05, device="cuda")
        q8 = torch.empty(t, h, device="cuda", dtype=torch.float8_e4m3fn)
        nbytes = t * h * 2 * 3 + t * h + h * 2
        us = self.us([lambda: ext.fused_add_rms_norm_static_fp8_quant(q8, x, r, w, scale, EPS)])
        cmp = {}
        if vllm is not None:
            cmp = self.comparators({"vllm": lambda: [
                lambda: vllm[0].fused_add_rms_norm_static_fp8_quant(q8, x, r, w, scale, EPS)]})
        self.put("ext fused add + RMSNorm + static fp8, 65536x8192", us, nbytes, cmp=cmp)
        del q8
        gscale = torch.full((1,), 448.0 * 6.0 / 8.0, device="cuda")
        q4 = torch.empty(t, h // 2, device="cuda", dtype=torch.uint8)
        sc = torch.empty(ext.nvfp4_scale_bytes(t, h), device="cuda", dtype=torch.uint8)
        nbytes = t * h * 2 * 3 + t * h // 2 + t * h // 16 + h * 2
        us = self.us([lambda: ext.rms_norm_nvfp4_quant(q4, sc, x, w, gscale, EPS, r)])
        cmp = {}
        if vllm is not None:
            sc32 = sc.view(torch.int32)

            def theirs():
                vllm[0].fused_add_rms_norm(x, r, w, EPS)
                vllm[0].scaled_fp4_quant.out(x, gscale, True, output=q4, output_scale=sc32)

            cmp = self.comparators({"vllm_fused_add_rms_norm_and_scaled_fp4_quant":
                                    lambda: [theirs]})
        self.put("ext fused add + RMSNorm + NVFP4 (tiled scales), 65536x8192", us, nbytes,
                 cmp=cmp)
        del x, r, q4, sc
        torch.cuda.empty_cache()

    def run(self, headline_us: float, headline_t1):
        d = self.dist
        self.rms_fp32()
        self.sweep()
        if self.cmp_on:
            us, nbytes, cmp = self.fused_add_comparators(1024, 4096)
            self.put("fused_add bf16 1024x4096 (dominant sweep call)", us, nbytes, cmp=cmp)
        self.qk_kv("qk_kv decode bf16 B=1 16/8", 1, 16, 8, 2048, False, sharded=False)
        for b in (64, 256, 1024):
            self.qk_kv(f"qk_kv decode bf16 B={b} 32/8", b, 32, 8, 65536, False, sharded=True)
        self.qk_kv("qk_kv prefill bf16 32768 tokens 64/8", 32768, 64, 8, 2048, True,
                   sharded=True)
        self.qk_no_kv()
        cmp = None
        if self.cmp_on:
            _, _, cmp = self.fused_add_comparators(HEADLINE_ROWS, HEADLINE_HIDDEN)
        self.put("fused_add prefill bf16 65536x8192 (headline)", headline_us,
                 fused_bytes(HEADLINE_ROWS, HEADLINE_HIDDEN, 2), sharded=True, t1=headline_t1,
                 cmp=cmp)
        if self.cmp_on:
            self.engine_formats()
        return self.out


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def repeat_child(args) -> None:
    """One process of the repeat protocol: the headline on one GPU,
    REPEAT_SAMPLES samples of `steps` timed steps each; prints the samples."""
    import sm120_rmsnorm as ops

    torch.cuda.set_device(0)
    head = PrefillRows(HEADLINE_ROWS, seed=1234)
    samples = [headline_step_ms(ops, head, args.steps, args.warmup, _solo())
               for _ in range(REPEAT_SAMPLES)]
    print(json.dumps({"samples_ms": samples}))


def spawn_repeats(extra_args: list[str], timeout: float) -> list[dict]:
    """Run REPEAT_PROCESSES independent child processes of this script and
    collect their JSON lines (the reference's run_repeated.py protocol)."""
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK",
                        "ROLE_RANK", "TORCHELASTIC_RUN_ID", "MASTER_ADDR", "MASTER_PORT")}
    results = []
    for _ in range(REPEAT_PROCESSES):
        proc = subprocess.run([sys.executable, str(Path(__file__).resolve()), *extra_args],
                              capture_output=True, text=True, env=env, timeout=timeout)
        if proc.returncode != 0:
            raise RuntimeError(f"repeat process failed (rc {proc.returncode}): "
                               f"{(proc.stderr or proc.stdout)[-400:]}")
        results.append(json.loads(proc.stdout.strip().splitlines()[-1]))
    return results


def repeat_summary(values: list[float], unit: str) -> dict:
    med = statistics.median(values)
    return {"processes": len(values), "median": round(med, 3), "unit": unit,
            "range_pct": round(100.0 * (max(values) - min(values)) / med, 2),
            "per_process": [round(v, 3) for v in values]}


def gpu_arm(args, dist: "Dist") -> dict:
    import sm120_rmsnorm as ops

    peak, peak_source = measured_hbm_peak()
    start, stop = shard_bounds(HEADLINE_ROWS, dist.world, dist.rank)
    head = PrefillRows(stop - start, seed=1234 + dist.rank)
    clocks = ClockSampler(sampled_gpus(dist.world) if dist.rank == 0 else None)
    with clocks:
        step_ms = headline_step_ms(ops, head, args.steps, args.warmup, dist)
        step_ms_max = dist.max(step_ms)
        if args.step_only:  # the timed steps alone (for a launch-list capture)
            return {"metric": "step only", "ms_per_step": round(step_ms_max, 5),
                    "gpu_launches": args.steps}
        line = _measure_rest(args, dist, ops, head, step_ms_max, peak, peak_source)
    line["clocks"] = clocks.summary() if dist.rank == 0 else None
    # `roofline` (with the per-config table) last, so a truncated tail keeps it
    line["roofline"] = line.pop("roofline")
    return line


def _measure_rest(args, dist, ops, head, step_ms_max, peak, peak_source) -> dict:
    total_bytes = fused_bytes(HEADLINE_ROWS, HEADLINE_HIDDEN, 2)
    value = total_bytes / (step_ms_max * 1e-3) / 1e9
    launch_us = step_ms_max * 1e3  # one launch per step on each rank
    achieved = head.bytes / (launch_us * 1e-6) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": dram_traffic_per_launch(head.rows),
                "kernel": f"fused_add_rms_norm_inplace bf16 {head.rows}x{HEADLINE_HIDDEN} "
                          "(one launch per step on each GPU; the slowest rank's)",
                "timing": "CUDA events around the timed steps on the launching stream; "
                          "launch duration = step time",
                "algorithmic_bytes_per_launch": head.bytes, "launch_us": round(launch_us, 2),
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of a "
                                  "smaller launch of the same kernel, scaled by rows "
                                  "(profiles/dram_traffic.txt)",
                "peak_source": peak_source + (", of measured" if peak_source.startswith("measured")
                                              else ", of fallback")}

    e2e = e2e_headline(ops, head, args.steps, dist)

    # whole problem on one GPU, for the headline's strong-scaling entry
    headline_t1 = None
    if dist.world > 1:
        dist.barrier()
        t1 = 0.0
        if dist.rank == 0:
            whole = PrefillRows(HEADLINE_ROWS, seed=1234)
            t1 = headline_step_ms(ops, whole, args.steps, args.warmup, _solo()) * 1e3
            del whole
            torch.cuda.empty_cache()
        dist.barrier()
        headline_t1 = dist.max(t1)

    flush = Flusher()
    per_config = {} if args.skip_per_config else PerConfig(ops, flush, dist, args, peak).run(
        launch_us, headline_t1)
    del flush
    torch.cuda.empty_cache()

    if dist.world == 1 and not args.skip_repeat:
        runs = spawn_repeats(["--repeat-child", "--steps", str(args.steps),
                              "--warmup", str(args.warmup)], timeout=600)
        per_process = [statistics.median(r["samples_ms"]) for r in runs]
        rep = repeat_summary([total_bytes / (ms * 1e-3) / 1e9 for ms in per_process], "GB/s")
        rep["ms_per_step_per_process"] = [round(ms, 4) for ms in per_process]
        rep["protocol"] = (f"{REPEAT_PROCESSES} independent processes x {REPEAT_SAMPLES} samples "
                           f"of {args.steps} timed steps (after {args.warmup} warm-up steps); "
                           "median of the per-process medians")
        roofline["repeat"] = rep
    roofline["per_config"] = per_config

    if args.detail:
        detail = {}
        flush = Flusher()
        detail["extensions"] = extension_suite(flush, dist, args)
        detail["engine"] = engine_suite(flush, dist, args)
        detail["projection"] = projection_suite(flush, dist, args)
        del flush
        if dist.rank == 0:
            Path(args.detail).parent.mkdir(parents=True, exist_ok=True)
            Path(args.detail).write_text(json.dumps(detail, indent=1))

    return {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms_max, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(1,0.1) weights)",
        "gpu_launches": args.steps,
        "config": {"workload": HEADLINE_WORKLOAD, "rows": HEADLINE_ROWS,
                   "hidden": HEADLINE_HIDDEN, "rows_per_gpu": head.rows,
                   "bytes_per_step": total_bytes,
                   "parallelism": f"rows sharded over {dist.world} GPU(s), no collective on the "
                                  "data path (NCCL only for barriers and the max-over-ranks time)",
                   "l2": "not flushed: each rank's x + residual (2 GiB / N) exceeds L2; the "
                         "per-config table flushes L2 (512 MiB write) before every timing"},
        "e2e": e2e, "roofline": roofline, "device": torch.cuda.get_device_name(),
    }


def _solo() -> "Dist":
    solo = Dist.__new__(Dist)
    solo.world, solo.rank, solo.local_rank, solo.pg = 1, 0, 0, None
    return solo


# ---------------------------------------------------------------------------
# detail suites (--detail): the engine-side extensions, the engine step and the
# QKV projection beside library comparators
# ---------------------------------------------------------------------------
def qk_cache_bytes(t: int, hq: int, hk: int, s: int, d: int = 128, rotary: int = 128,
                   cache_elem: int | None = None) -> int:
    # as qk_kv_bytes, with the two cache stores at the cache element size
    cache_elem = s if cache_elem is None else cache_elem
    return (t * (s * d * (2 * hq + 3 * hk) + 2 * cache_elem * d * hk + 8 + 4 + 4 * rotary)
            + 2 * d * s)


def norm_quant_bytes(t: int, h: int, s: int, add: bool, dynamic: bool) -> int:
    # x read (and r read + written), fp8 result written, weight once, scales
    return t * h * s * (3 if add else 1) + t * h + h * s + (4 * t if dynamic else 0)


def extension_suite(flush: Flusher, dist: Dist, args) -> dict:
    """The engine-side extensions (sm120_rmsnorm.extensions) at decode and
    prefill shapes, each beside the unfused vLLM pair that does the same work
    when vLLM's kernels load (timed the same way: graphs of back-to-back calls
    on distinct buffer sets after an L2 flush)."""
    from sm120_rmsnorm import extensions as ext

    out = {}
    reps = max(3, args.reps)
    g = torch.Generator(device="cuda").manual_seed(123 + dist.rank)
    cpu_g = torch.Generator().manual_seed(17 + dist.rank)
    bf = torch.bfloat16
    vllm = vllm_ops()

    def sets_for(nbytes):
        return max(1, min(64, (256 << 20) // max(nbytes, 1)))

    def record(name, calls, nbytes, **extra):
        try:
            graph, _ = capture(calls)
            us = dist.max(time_graph(graph, flush, reps) / len(calls))
            out[name] = {"us": round(us, 3), "bytes": nbytes,
                         "gbs": round(nbytes / (us * 1e-6) / 1e9, 1), **extra}
            del graph
        except Exception as e:  # noqa: BLE001 - only comparators may fail here
            if not extra.get("comparator"):
                raise
            out[name] = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
            torch.cuda.synchronize()

    def table(n, rotary=128, dtype=torch.float32):
        inv = 1.0 / (1e6 ** (torch.arange(0, rotary, 2, dtype=torch.float32, device="cuda") / rotary))
        f = torch.outer(torch.arange(n, dtype=torch.float32, device="cuda"), inv)
        return torch.cat((f.cos(), f.sin()), dim=-1).to(dtype)

    cache32, cache_bf = table(32768), table(32768, dtype=bf)
    one = torch.ones(1, device="cuda")
    qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
    kw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)

    def qk_cache_case(name, b, hq, hk, blocks, layout, fp8, contiguous, strided):
        cache_dtype = torch.float8_e4m3fn if fp8 else bf
        nbytes = qk_cache_bytes(b, hq, hk, 2, cache_elem=1 if fp8 else 2)
        n_sets = sets_for(nbytes)
        shape = (blocks, 16, hk, 128) if layout == "NHD" else (blocks, hk, 16, 128)
        kc = torch.zeros(shape, device="cuda", dtype=cache_dtype)
        vc = torch.zeros_like(kc)
        all_slots = torch.randperm(blocks * 16, generator=cpu_g)[: b * n_sets].to(torch.int32)
        sets = []
        for i in range(n_sets):
            qkv = torch.randn(b, (hq + 2 * hk) * 128, device="cuda", generator=g).to(bf)
            if contiguous:
                pos = torch.arange(b, device="cuda")
                slots = torch.arange(b, device="cuda", dtype=torch.int32)
            else:
                pos = torch.randperm(32768, generator=cpu_g)[:b].cuda()
                slots = all_slots[i * b:(i + 1) * b].cuda()
            if strided:
                q = qkv[:, :hq * 128].view(b, hq, 128)
                k = qkv[:, hq * 128:(hq + hk) * 128].view(b, hk, 128)
                v = qkv[:, (hq + hk) * 128:].view(b, hk, 128)
            else:
                q = qkv[:, :hq * 128].reshape(b, hq, 128).contiguous()
                k = qkv[:, hq * 128:(hq + hk) * 128].reshape(b, hk, 128).contiguous()
                v = qkv[:, (hq + hk) * 128:].reshape(b, hk, 128).contiguous()
            sets.append((qkv, q, k, v, pos, slots))
        scales = (one, one) if fp8 else (None, None)
        calls = [lambda q=q, k=k, v=v, pos=pos, slots=slots: ext.qk_norm_rope_cache_(
            q, k, v, qw, kw, pos, cache32, kc, vc, slots, *scales, True, layout, EPS)
            for (_, q, k, v, pos, slots) in sets]
        record(name, calls, nbytes)
        if vllm is not None and strided and layout == "NHD":
            C, cache_ops = vllm
            kv_dtype = "fp8" if fp8 else "auto"
            vkc = torch.zeros((blocks, 16, hk, 128), device="cuda",
                              dtype=torch.uint8 if fp8 else bf)
            vvc = torch.zeros_like(vkc)

            def unfused(qkv, k, v, pos, slots):
                C.fused_qk_norm_rope(qkv, hq, hk, hk, 128, EPS, qw, kw, cache_bf, True, pos)
                cache_ops.reshape_and_cache_flash(k, v, vkc, vvc, slots.long(), kv_dtype, one, one)

            calls = [lambda qkv=qkv, k=k, v=v, pos=pos, slots=slots: unfused(qkv, k, v, pos, slots)
                     for (qkv, _, k, v, pos, slots) in sets]
            record(name + " [vLLM fused_qk_norm_rope + reshape_and_cache_flash]", calls, nbytes,
                   comparator=True)
        del sets, kc, vc

    qk_cache_case("qk_cache decode bf16 B=1024 32/8 strided qkv, fp8 NHD cache",
                  1024, 32, 8, 65536, "NHD", True, False, True)
    qk_cache_case("qk_cache decode bf16 B=1024 32/8 strided qkv, bf16 NHD cache",
                  1024, 32, 8, 65536, "NHD", False, False, True)
    qk_cache_case("qk_cache decode bf16 B=1 16/8 strided qkv, fp8 NHD cache",
                  1, 16, 8, 2048, "NHD", True, False, True)
    qk_cache_case("qk_cache prefill bf16 32768 tokens 64/8 strided qkv, bf16 NHD cache",
                  32768, 64, 8, 2048, "NHD", False, True, True)
    qk_cache_case("qk_cache prefill bf16 32768 tokens 64/8 strided qkv, fp8 NHD cache",
                  32768, 64, 8, 2048, "NHD", True, True, True)
    qk_cache_case("qk_cache prefill bf16 32768 tokens 64/8, bf16 HND cache",
                  32768, 64, 8, 2048, "HND", False, True, False)

    # RMSNorm + fp8 quantisation
    def quant_case(name, t, h, add, dynamic):
        nbytes = norm_quant_bytes(t, h, 2, add, dynamic)
        w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(bf)
        scale = torch.full((1,), 0.05, device="cuda")
        sets = []
        for _ in range(sets_for(nbytes)):
            x = torch.randn(t, h, device="cuda", generator=g).to(bf)
            r = torch.randn(t, h, device="cuda", generator=g).to(bf) if add else None
            res = torch.empty(t, h, device="cuda", dtype=torch.float8_e4m3fn)
            scales = torch.empty(t, device="cuda") if dynamic else None
            sets.append((x, r, res, scales))

        def ours(x, r, res, scales):
            if dynamic:
                ext.rms_norm_dynamic_per_token_quant(res, x, w, scales, EPS, None, r)
            elif add:
                ext.fused_add_rms_norm_static_fp8_quant(res, x, r, w, scale, EPS)
            else:
                ext.rms_norm_static_fp8_quant(res, x, w, scale, EPS)

        record(name, [lambda s=s: ours(*s) for s in sets], nbytes)
        if vllm is not None:
            C, _ = vllm

            def theirs(x, r, res, scales):
                if dynamic:
                    C.rms_norm_dynamic_per_token_quant(res, x, w, scales.view(-1, 1), EPS, None, r)
                elif add:
                    C.fused_add_rms_norm_static_fp8_quant(res, x, r, w, scale, EPS)
                else:
                    C.rms_norm_static_fp8_quant(res, x, w, scale, EPS)

            record(name + " [vLLM]", [lambda s=s: theirs(*s) for s in sets], nbytes,
                   comparator=True)
        del sets

    quant_case("fused_add_rms_norm_static_fp8_quant bf16 1024x4096", 1024, 4096, True, False)
    quant_case("rms_norm_dynamic_per_token_quant bf16 1024x4096", 1024, 4096, False, True)
    quant_case("rms_norm_dynamic_per_token_quant + residual bf16 1024x4096", 1024, 4096, True, True)
    quant_case("fused_add_rms_norm_static_fp8_quant prefill bf16 65536x8192", 65536, 8192, True,
               False)

    # RMSNorm + NVFP4 (e2m1 values, e4m3 scales per 16 elements, tiled scales)
    def fp4_case(name, t, h):
        nbytes = t * h * 2 * 3 + t * h // 2 + t * h // 16 + h * 2
        w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(bf)
        gscale = torch.full((1,), 448.0 * 6.0 / 8.0, device="cuda")
        sets = []
        for _ in range(sets_for(nbytes)):
            x = torch.randn(t, h, device="cuda", generator=g).to(bf)
            r = torch.randn(t, h, device="cuda", generator=g).to(bf)
            q = torch.empty(t, h // 2, device="cuda", dtype=torch.uint8)
            sc = torch.empty(ext.nvfp4_scale_bytes(t, h), device="cuda", dtype=torch.uint8)
            sets.append((x, r, q, sc))
        record(name, [lambda s=s: ext.rms_norm_nvfp4_quant(s[2], s[3], s[0], w, gscale, EPS, s[1])
                      for s in sets], nbytes)
        if vllm is not None:
            C, _ = vllm
            scale_i32 = [torch.empty(sc.numel() // 4, device="cuda", dtype=torch.int32)
                         for (_, _, _, sc) in sets]

            def theirs(x, r, q, sc32):
                C.fused_add_rms_norm(x, r, w, EPS)
                C.scaled_fp4_quant.out(x, gscale, True, output=q, output_scale=sc32)

            record(name + " [vLLM fused_add_rms_norm + scaled_fp4_quant]",
                   [lambda s=s, sc32=sc32: theirs(s[0], s[1], s[2], sc32)
                    for s, sc32 in zip(sets, scale_i32)], nbytes, comparator=True)
        del sets

    fp4_case("fused add + rms_norm_nvfp4_quant bf16 1024x4096", 1024, 4096)
    fp4_case("fused add + rms_norm_nvfp4_quant prefill bf16 65536x8192", 65536, 8192)

    # the headline op beside vLLM's and FlashInfer's residual add + RMSNorm on
    # the same shapes (library comparators: timed here, never on the product path)
    import sm120_rmsnorm as ops
    flashinfer_norm = flashinfer_fused_add_rmsnorm()
    for t, h in ((1024, 4096), (65536, 8192)):
        nbytes = fused_bytes(t, h, 2)
        w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(bf)
        sets = [(torch.randn(t, h, device="cuda", generator=g).to(bf),
                 torch.randn(t, h, device="cuda", generator=g).to(bf))
                for _ in range(sets_for(nbytes))]
        record(f"fused_add_rms_norm_inplace bf16 {t}x{h}",
               [lambda x=x, r=r: ops.fused_add_rms_norm_inplace(x, r, w, EPS) for x, r in sets],
               nbytes)
        if vllm is not None:
            C, _ = vllm
            record(f"fused_add_rms_norm_inplace bf16 {t}x{h} [vLLM fused_add_rms_norm]",
                   [lambda x=x, r=r: C.fused_add_rms_norm(x, r, w, EPS) for x, r in sets],
                   nbytes, comparator=True)
        if flashinfer_norm is not None:
            record(f"fused_add_rms_norm_inplace bf16 {t}x{h} [FlashInfer fused_add_rmsnorm]",
                   [lambda x=x, r=r: flashinfer_norm(x, r, w, EPS) for x, r in sets],
                   nbytes, comparator=True)
        del sets
    out["flashinfer_comparator"] = "loaded" if flashinfer_norm is not None else "unavailable"
    out["vllm_comparator"] = "loaded" if vllm is not None else "unavailable"
    return out


def engine_suite(flush: Flusher, dist: Dist, args) -> dict:
    """Decode-step attention prologues of a Qwen3-8B-shaped model (hidden 4096,
    32 query / 8 KV heads of 128, bf16, random weights): for each of L layers
    residual add + input RMSNorm, the QKV projection (cuBLAS through PyTorch),
    Q/K norm + RoPE + paged KV store; L layers captured in one CUDA graph per
    path and batch, replayed after an L2 flush. Paths: this package
    (sm120_rmsnorm.engine.DecodeGraph: 2 own kernels per layer, in place on the
    QKV buffer), the reference's kernels (contiguous Q / K / V copies first,
    as its operator requires), and vLLM's kernels when they load. `gemm_only`
    is the projection plus the stand-in copy between layers, so
    `norm_us_per_layer` = (path - gemm_only) / L is the per-layer cost of the
    normalisation path itself."""
    from oracle import build_ref
    from sm120_rmsnorm.engine import (DecodeGraph, Qwen3AttentionPrologue, Qwen3AttentionShape,
                                      rope_cos_sin_cache)

    shape = Qwen3AttentionShape()
    n_layers = 8
    reps = max(3, args.reps)
    bf = torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(31 + dist.rank)
    cpu_g = torch.Generator().manual_seed(37 + dist.rank)
    layers = [Qwen3AttentionPrologue(shape, "cuda", generator=g) for _ in range(n_layers)]
    cos_sin = rope_cos_sin_cache(shape, "cuda")
    cos_bf = cos_sin.to(bf)
    ref = build_ref.load()
    vllm = vllm_ops()
    one = torch.ones(1, device="cuda")
    out = {"model": "Qwen3-8B-shaped attention prologue (hidden 4096, 32/8 heads x 128, bf16)",
           "layers": n_layers}

    def time_graph_us(graph):
        return dist.max(time_graph(graph, flush, reps))

    def generic_graph(batch, positions, slots, kcs, vcs, prologue):
        hidden = torch.randn(batch, shape.hidden, device="cuda", generator=g).to(bf)
        residual = torch.randn(batch, shape.hidden, device="cuda", generator=g).to(bf)
        qkvs = [torch.empty(batch, shape.qkv_width, device="cuda", dtype=bf) for _ in layers]
        nexts = [torch.empty_like(hidden) for _ in layers[1:]]

        def run():
            h = hidden
            for i, layer in enumerate(layers):
                prologue(layer, h, residual, positions, slots, kcs[i], vcs[i], qkvs[i])
                if i + 1 < len(layers):
                    nexts[i].copy_(qkvs[i][:, :shape.hidden])
                    h = nexts[i]
        graph, _ = capture([run])
        return graph

    def gemm_only(layer, h, r, pos, slots, kc, vc, qkv):
        torch.matmul(h, layer.qkv_weight.t(), out=qkv)

    def reference_path(layer, h, r, pos, slots, kc, vc, qkv):
        ref.fused_add_rms_norm_inplace(h, r, layer.input_norm_weight, EPS, 0)
        torch.matmul(h, layer.qkv_weight.t(), out=qkv)
        q, k, v = (t.contiguous() for t in layer.split(qkv))
        ref.fused_qk_rms_norm_rope_kv(q, k, v, layer.query_norm_weight, layer.key_norm_weight,
                                      pos, cos_sin, kc, vc, slots, EPS, 1)

    def vllm_path(layer, h, r, pos, slots, kc, vc, qkv):
        C, cache_ops = vllm
        C.fused_add_rms_norm(h, r, layer.input_norm_weight, EPS)
        torch.matmul(h, layer.qkv_weight.t(), out=qkv)
        C.fused_qk_norm_rope(qkv, shape.query_heads, shape.key_heads, shape.key_heads,
                             shape.head_dim, EPS, layer.query_norm_weight, layer.key_norm_weight,
                             cos_bf, True, pos)
        _, k, v = layer.split(qkv)
        cache_ops.reshape_and_cache_flash(k, v, kc, vc, slots.long(), "auto", one, one)

    for batch in (1, 64, 256):
        blocks = max(64, 4 * batch // 16)
        kcs = [torch.zeros(blocks, 16, shape.key_heads, shape.head_dim, device="cuda", dtype=bf)
               for _ in layers]
        vcs = [torch.zeros_like(kc) for kc in kcs]
        positions = torch.randperm(shape.max_positions, generator=cpu_g)[:batch].cuda()
        slots = torch.randperm(blocks * 16, generator=cpu_g)[:batch].to(torch.int32).cuda()
        row = {}
        ours = DecodeGraph(layers, batch, cos_sin, kcs, vcs, fused_projection=False)
        ours.hidden.copy_(torch.randn(batch, shape.hidden, device="cuda", generator=g).to(bf))
        ours.residual.copy_(torch.randn(batch, shape.hidden, device="cuda", generator=g).to(bf))
        ours.positions.copy_(positions)
        ours.slot_mapping.copy_(slots)
        row["b200"] = time_graph_us(ours.graph)
        del ours
        fused = DecodeGraph(layers, batch, cos_sin, kcs, vcs, fused_projection=True)
        fused.hidden.copy_(torch.randn(batch, shape.hidden, device="cuda", generator=g).to(bf))
        fused.residual.copy_(torch.randn(batch, shape.hidden, device="cuda", generator=g).to(bf))
        fused.positions.copy_(positions)
        fused.slot_mapping.copy_(slots)
        row["b200_fused_projection"] = time_graph_us(fused.graph)
        del fused
        base = generic_graph(batch, positions, slots, kcs, vcs, gemm_only)
        row["gemm_only"] = time_graph_us(base)
        del base
        if ref is not None:
            graph = generic_graph(batch, positions, slots, kcs, vcs, reference_path)
            row["reference_kernels"] = time_graph_us(graph)
            del graph
        if vllm is not None:
            try:
                graph = generic_graph(batch, positions, slots, kcs, vcs, vllm_path)
                row["vllm"] = time_graph_us(graph)
                del graph
            except Exception as e:  # noqa: BLE001 - a comparator may be unavailable
                row["vllm_unavailable"] = f"{type(e).__name__}: {str(e)[:160]}"
                torch.cuda.synchronize()
        entry = {"us_per_step": {k: round(v, 2) for k, v in row.items()
                                 if isinstance(v, float)}}
        entry["norm_us_per_layer"] = {
            k: round((v - row["gemm_only"]) / n_layers, 3) for k, v in row.items()
            if isinstance(v, float) and k != "gemm_only"}
        if "vllm_unavailable" in row:
            entry["vllm_unavailable"] = row["vllm_unavailable"]
        out[f"decode B={batch}"] = entry
        del kcs, vcs
    return out


def projection_suite(flush: Flusher, dist: Dist, args) -> dict:
    """The QKV projection of a Qwen3-8B-shaped layer (hidden 4096, 32/8 heads
    of 128, bf16) at decode and prefill token counts: this package's
    tensor-core GEMM alone and with the Q/K norm + RoPE + KV store fused into
    its epilogue, against PyTorch's GEMM (cuBLAS) alone and followed by the
    stand-alone Q/K kernel on the strided QKV views -- the unfused path the
    fusion replaces. Same protocol as the other suites; TFLOP/s counts the
    GEMM's 2 * T * N * K."""
    from sm120_rmsnorm import extensions as ext

    out = {}
    reps = max(3, args.reps)
    bf = torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(41 + dist.rank)
    hidden, hq, hk = 4096, 32, 8
    n = (hq + 2 * hk) * 128
    w = (torch.randn(n, hidden, device="cuda", generator=g) / hidden ** 0.5).to(bf)
    qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
    kw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
    f = torch.outer(torch.arange(32768, dtype=torch.float32, device="cuda"), inv)
    table = torch.cat((f.cos(), f.sin()), dim=-1)
    for t in (1, 64, 256, 4096, 32768):
        x = torch.randn(t, hidden, device="cuda", generator=g).to(bf)
        qkv = torch.empty(t, n, device="cuda", dtype=bf)
        pos = torch.randint(0, 32768, (t,), device="cuda", generator=g)
        slots_total = max(4 * t, 4096)
        slots = torch.randperm(slots_total, device="cuda", generator=g)[:t].to(torch.int32)
        kc = torch.zeros(slots_total, hk, 128, device="cuda", dtype=bf)
        vc = torch.zeros_like(kc)
        views = (qkv[:, :hq * 128].view(t, hq, 128), qkv[:, hq * 128:(hq + hk) * 128].view(t, hk, 128),
                 qkv[:, (hq + hk) * 128:].view(t, hk, 128))
        flops = 2.0 * t * n * hidden
        cases = {
            "cublas_gemm": lambda: torch.matmul(x, w.t(), out=qkv),
            "own_gemm": lambda: ext.qkv_proj_norm_rope_cache_(x, w, qkv, hq, hk, fuse_norm=False),
            "cublas_gemm_then_qk_kernel": lambda: (
                torch.matmul(x, w.t(), out=qkv),
                ext.qk_norm_rope_cache_(views[0], views[1], views[2], qw, kw, pos, table,
                                        kc.view(-1, 1, hk, 128), vc.view(-1, 1, hk, 128),
                                        slots)),
            "fused_projection": lambda: ext.qkv_proj_norm_rope_cache_(
                x, w, qkv, hq, hk, qw, kw, pos, table, kc, vc, slots),
        }
        entry = {}
        for name, fn in cases.items():
            graph, _ = capture([fn])
            us = dist.max(time_graph(graph, flush, reps))
            entry[name] = {"us": round(us, 2), "tflops": round(flops / (us * 1e-6) / 1e12, 1)}
            del graph
        out[f"tokens={t}"] = entry
        del x, qkv, kc, vc
    return out


# ---------------------------------------------------------------------------
# CPU arms (the oracle is the checker and the CPU baseline, nothing else)
# ---------------------------------------------------------------------------
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_rows(rows: int, seed: int):
    """x, residual [rows, 8192] bf16 and the weight on the host, drawn from
    N(0,1) / N(1,0.1): one seeded 2048-row block repeated down the rows (the
    CPU's caches hold far less than a block, so the timing is that of the
    full-size arrays; drawing 2^29 normals would take longer than the timing)."""
    g = torch.Generator().manual_seed(seed)
    block = min(rows, 2048)
    h = HEADLINE_HIDDEN
    xb = torch.randn(block, h, generator=g).to(torch.bfloat16)
    rb = torch.randn(block, h, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16)
    reps = (rows + block - 1) // block
    x = xb.repeat(reps, 1)[:rows].contiguous()
    r = rb.repeat(reps, 1)[:rows].contiguous()
    return x, r, w


def cpu_port_timing(rows: int, threads: int, calls: int | None, seconds: float,
                    warmup: int = 1):
    """The C restatement of the reference's CPU path, in place on [rows, 8192]
    bf16 host arrays: `warmup` untimed calls, then `calls` timed calls (or as
    many as fit in `seconds`). Returns (GB/s, calls, elapsed s, per-call s)."""
    from oracle import oracle

    oracle.build()
    oracle.set_threads(threads)
    x, r, w = cpu_rows(rows, seed=4321)
    nbytes = fused_bytes(rows, HEADLINE_HIDDEN, 2)
    for _ in range(warmup):
        oracle.fused_add_rms_norm_out(x, r, w, x, r, EPS)
    per_call = []
    t0 = time.perf_counter()
    while True:
        c0 = time.perf_counter()
        oracle.fused_add_rms_norm_out(x, r, w, x, r, EPS)
        per_call.append(time.perf_counter() - c0)
        elapsed = time.perf_counter() - t0
        if (calls is not None and len(per_call) >= calls) or (calls is None and elapsed >= seconds):
            break
    return nbytes * len(per_call) / elapsed / 1e9, len(per_call), elapsed, per_call


def reference_child(args) -> None:
    """One process of the reference arm: the headline workload through the C
    restatement of the reference's CPU path on all host threads."""
    threads = host_threads()
    gbs, calls, elapsed, per_call = cpu_port_timing(HEADLINE_ROWS, threads, args.steps, 0,
                                                    warmup=args.warmup)
    print(json.dumps({"gbs": gbs, "calls": calls, "elapsed_s": elapsed,
                      "ms_per_step": elapsed / calls * 1e3, "threads": threads}))


def reference_kernels_gpu(args) -> dict:
    """The reference's CUDA kernels on this B200 on the headline workload
    (the SM120 kernels rebuilt for sm_100a: the bar to beat), same steps and
    warm-up as the GPU arm."""
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    ref = ReferenceKernels.load()
    if ref is None:
        return {"unavailable": "the reference's kernels were not built (oracle/build_ref.py "
                               "needs the reference checkout)"}
    torch.cuda.set_device(0)
    head = PrefillRows(HEADLINE_ROWS, seed=1234)
    ms = headline_step_ms(ref, head, args.steps, args.warmup, _solo())
    return {"value": round(head.bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(ms, 4), "steps": args.steps, "warmup": args.warmup,
            "build": "reference csrc/rmsnorm_kernels.cu + bindings.cpp, nvcc -O3 "
                     "--use_fast_math -gencode arch=compute_100a,code=sm_100a",
            "call": "fused_add_rms_norm_inplace(x, residual, weight, 1e-6, version=0)"}


def pytorch_cpu_reference(threads: int, rows: int = 2048, calls: int = 5) -> dict:
    """The reference's PyTorch oracle math (residual add + RMSNorm,
    reference.py:14-24 in the reference project; restated op for op in
    sm120_rmsnorm/reference.py, loaded by file path so nothing else of the
    package is imported) on the host CPU, on a bounded sample of the rows."""
    import importlib.util

    path = ROOT / "sm120-norm-fusion-kernels_b200" / "sm120_rmsnorm" / "reference.py"
    spec = importlib.util.spec_from_file_location("sweep_reference_math", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    torch.set_num_threads(threads)
    x, r, w = cpu_rows(rows, seed=4321)
    module.fused_add_rms_norm_reference(x, r, w, EPS)
    t0 = time.perf_counter()
    for _ in range(calls):
        module.fused_add_rms_norm_reference(x, r, w, EPS)
    elapsed = time.perf_counter() - t0
    return {"value": round(fused_bytes(rows, HEADLINE_HIDDEN, 2) * calls / elapsed / 1e9, 3),
            "unit": "GB/s", "threads": threads,
            "sample": f"{calls} calls on {rows} of the 65536 rows, {elapsed:.2f} s"}


def pytorch_cpu_per_config(threads: int) -> dict:
    """The reference's PyTorch math (restated op for op in
    sm120_rmsnorm/reference.py) on the host CPU for the small configurations,
    as the reference's own CPU baseline measures them: per call, after a
    warm-up call, at least 200 calls or 20 ms (time.perf_counter), all host
    threads; keyed like the GPU arm's per-config entries, with GB/s from the
    same byte formulas. The Q/K-KV decode includes the two paged-cache stores."""
    import importlib.util

    path = ROOT / "sm120-norm-fusion-kernels_b200" / "sm120_rmsnorm" / "reference.py"
    spec = importlib.util.spec_from_file_location("config_reference_math", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(97)

    def per_call_us(fn):
        fn()
        calls, t0 = 0, time.perf_counter()
        while calls < 200 or time.perf_counter() - t0 < 0.02:
            fn()
            calls += 1
            if calls >= 200 and time.perf_counter() - t0 >= 0.02:
                break
        return (time.perf_counter() - t0) / calls * 1e6

    out = {}

    def put(name, us, nbytes):
        out[name] = {"us": round(us, 2), "gbs": round(nbytes / (us * 1e-6) / 1e9, 3)}

    for t in (1, 4, 16, 64, 256):
        x = torch.randn(t, 1024, generator=g)
        w = 1 + 0.1 * torch.randn(1024, generator=g)
        put(f"rms_norm fp32 {t}x1024", per_call_us(lambda: ref.rms_norm_reference(x, w, EPS)),
            rms_bytes(t, 1024, 4))
    step_us, step_bytes = 0.0, 0
    for t, h, name in sweep_shapes():
        dt = DTYPES[name]
        x = torch.randn(t, h, generator=g).to(dt)
        r = torch.randn(t, h, generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(h, generator=g)).to(dt)
        us = per_call_us(lambda: ref.fused_add_rms_norm_reference(x, r, w, EPS))
        step_us += us
        step_bytes += fused_bytes(t, h, 2)
        if (t, h, name) == (1024, 4096, "bf16"):
            put("fused_add bf16 1024x4096 (dominant sweep call)", us, fused_bytes(t, h, 2))
    put("fused_add sweep 48 calls (step)", step_us, step_bytes)
    cache = rope_table(32768, device="cpu")
    bf = torch.bfloat16
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(bf)
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(bf)
    q = torch.randn(1, 16, 128, generator=g).to(bf)
    k = torch.randn(1, 8, 128, generator=g).to(bf)
    v = torch.randn(1, 8, 128, generator=g).to(bf)
    pos = torch.randint(0, 32768, (1,), generator=g)
    slots = torch.randint(0, 2048 * 16, (1,), generator=g)
    kc = torch.zeros(2048 * 16, 8, 128, dtype=bf)
    vc = torch.zeros_like(kc)

    def qk_kv():
        qo, ko = ref.qk_rms_norm_rope_reference(q, k, qw, kw, pos, cache, EPS)
        kc[slots] = ko
        vc[slots] = v

    put("qk_kv decode bf16 B=1 16/8", per_call_us(qk_kv), qk_kv_bytes(1, 16, 8, 2))
    for t in (1, 4, 16, 64, 256):
        qt = torch.randn(t, 16, 128, generator=g).to(bf)
        kt = torch.randn(t, 8, 128, generator=g).to(bf)
        pt = torch.arange(t)
        put(f"qk (no kv) bf16 T={t} 16/8",
            per_call_us(lambda: ref.qk_rms_norm_rope_reference(qt, kt, qw, kw, pt, cache, EPS)),
            qk_bytes(t, 16, 8, 2))
    return out


def reference_arm(args) -> dict:
    """The reference path's CPU implementation (C restatement of its PyTorch
    oracle) on the host cores, on the headline workload, in REPEAT_PROCESSES
    independent processes of `steps` timed calls each; rank 0 only."""
    runs = spawn_repeats(["--impl", "reference", "--reference-child", "--steps",
                          str(args.steps), "--warmup", str(args.warmup)], timeout=900)
    values = [r["gbs"] for r in runs]
    rep = repeat_summary(values, "GB/s")
    value = rep["median"]
    ms = statistics.median(r["ms_per_step"] for r in runs)
    threads = runs[0]["threads"]
    timed = sum(r["elapsed_s"] for r in runs)
    sample = (f"the full workload, {args.steps} timed calls (after {args.warmup} warm-up calls) "
              f"in each of {REPEAT_PROCESSES} processes, {timed:.1f} s timed in all; median of "
              "the per-process GB/s")
    rep["protocol"] = sample
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": HEADLINE_WORKLOAD, "rows": HEADLINE_ROWS,
                   "hidden": HEADLINE_HIDDEN, "parallelism": f"{threads} host threads (OpenMP)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "repeat": rep,
        "note": "the reference's CPU path is its PyTorch oracle (sm120_rmsnorm/reference.py), "
                "which cannot travel; this is its C restatement (oracle/norm_oracle.c), pinned "
                "to the reference's own outputs by the golden-vector tests",
        "reference_pytorch_cpu": pytorch_cpu_reference(threads),
        "reference_pytorch_cpu_per_config": pytorch_cpu_per_config(threads),
        "reference_kernels_b200": reference_kernels_gpu(args),
    }


# ---------------------------------------------------------------------------
def profile_case(args) -> None:
    """Launch one operator at one shape `--launches` times (for ncu: skip the
    first launches with -s and capture one with -c 1)."""
    import sm120_rmsnorm as ops

    torch.cuda.set_device(0)
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[args.dtype]
    g = torch.Generator(device="cuda").manual_seed(0)
    t, h = args.tokens, args.hidden
    if args.profile in ("fused", "rms"):
        x = torch.randn(t, h, device="cuda", generator=g).to(dt)
        r = torch.randn(t, h, device="cuda", generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(dt)
        y = torch.empty_like(x)
        if args.profile == "fused":
            fn = lambda: ops.fused_add_rms_norm_inplace(x, r, w, EPS, args.version)
        else:
            fn = lambda: ops.rms_norm_out(x, w, y, EPS, args.version or 2)
    elif args.profile == "quant":
        from sm120_rmsnorm import extensions as ext
        x = torch.randn(t, h, device="cuda", generator=g).to(dt)
        r = torch.randn(t, h, device="cuda", generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(dt)
        out = torch.empty(t, h, device="cuda", dtype=torch.float8_e4m3fn)
        scale = torch.full((1,), 0.05, device="cuda")
        fn = lambda: ext.fused_add_rms_norm_static_fp8_quant(out, x, r, w, scale, EPS)
    elif args.profile == "fp4":
        from sm120_rmsnorm import extensions as ext
        x = torch.randn(t, h, device="cuda", generator=g).to(dt)
        r = torch.randn(t, h, device="cuda", generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(dt)
        out = torch.empty(t, h // 2, device="cuda", dtype=torch.uint8)
        scales = torch.empty(ext.nvfp4_scale_bytes(t, h), device="cuda", dtype=torch.uint8)
        gscale = torch.full((1,), 448.0 * 6.0 / 4.0, device="cuda")
        fn = lambda: ext.rms_norm_nvfp4_quant(out, scales, x, w, gscale, EPS, r)
    elif args.profile == "projection":
        from sm120_rmsnorm import extensions as ext
        hq, hk = (int(v) for v in args.heads.split(","))
        n = (hq + 2 * hk) * 128
        x = torch.randn(t, h, device="cuda", generator=g).to(dt)
        w = (torch.randn(n, h, device="cuda", generator=g) / h ** 0.5).to(dt)
        qkv = torch.empty(t, n, device="cuda", dtype=dt)
        qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(dt)
        inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
        f = torch.outer(torch.arange(32768, dtype=torch.float32, device="cuda"), inv)
        cache = torch.cat((f.cos(), f.sin()), dim=-1)
        pos = torch.randint(0, 32768, (t,), device="cuda")
        fn = lambda: ext.qkv_proj_norm_rope_cache_(x, w, qkv, hq, hk, qw, qw, pos, cache)
    elif args.profile == "qkcache":
        from sm120_rmsnorm import extensions as ext
        hq, hk = (int(v) for v in args.heads.split(","))
        qkv = torch.randn(t, (hq + 2 * hk) * 128, device="cuda", generator=g).to(dt)
        q = qkv[:, :hq * 128].view(t, hq, 128)
        k = qkv[:, hq * 128:(hq + hk) * 128].view(t, hk, 128)
        v = qkv[:, (hq + hk) * 128:].view(t, hk, 128)
        qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(dt)
        inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
        f = torch.outer(torch.arange(32768, dtype=torch.float32, device="cuda"), inv)
        cache = torch.cat((f.cos(), f.sin()), dim=-1)
        pos = torch.randint(0, 32768, (t,), device="cuda")
        blocks = max(t, 2048 * 16) // 16
        kc = torch.zeros(blocks, 16, hk, 128, device="cuda", dtype=torch.float8_e4m3fn)
        vc = torch.zeros_like(kc)
        slots = torch.randperm(blocks * 16, device="cuda")[:t].to(torch.int32)
        one = torch.ones(1, device="cuda")
        fn = lambda: ext.qk_norm_rope_cache_(q, k, v, qw, qw, pos, cache, kc, vc, slots, one, one)
    else:
        hq, hk = (int(v) for v in args.heads.split(","))
        q = torch.randn(t, hq, 128, device="cuda", generator=g).to(dt)
        k = torch.randn(t, hk, 128, device="cuda", generator=g).to(dt)
        v = torch.randn(t, hk, 128, device="cuda", generator=g).to(dt)
        qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(dt)
        inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
        f = torch.outer(torch.arange(32768, dtype=torch.float32, device="cuda"), inv)
        cache = torch.cat((f.cos(), f.sin()), dim=-1)
        pos = torch.randint(0, 32768, (t,), device="cuda")
        slots_total = max(t, 2048 * 16)
        kc = torch.zeros(slots_total, hk, 128, device="cuda", dtype=dt)
        vc = torch.zeros_like(kc)
        slots = torch.randperm(slots_total, device="cuda")[:t].to(torch.int32)
        if args.profile == "qkkv":
            fn = lambda: ops.fused_qk_rms_norm_rope_kv(q, k, v, qw, qw, pos, cache, kc, vc, slots,
                                                       EPS, args.version or 1)
        else:
            fn = lambda: ops.fused_qk_rms_norm_rope(q, k, qw, qw, pos, cache, EPS,
                                                    args.version or 2)
    flush = Flusher()
    for _ in range(args.launches):
        if not args.warm:  # --warm: inputs stay L2-resident, as in a decode loop
            flush()
        fn()
    torch.cuda.synchronize()
    print(f"profile: {args.profile} {args.dtype} tokens={t} hidden={h} heads={args.heads} "
          f"launches={args.launches}")


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--reps", type=int, default=10, help="replays per per-config timing")
    parser.add_argument("--impl", choices=["b200", "reference"], default="b200")
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--skip-per-config", action="store_true")
    parser.add_argument("--skip-comparators", action="store_true")
    parser.add_argument("--skip-cpu", action="store_true")
    parser.add_argument("--skip-repeat", action="store_true")
    parser.add_argument("--detail", help="also run the extension / engine / projection suites "
                                         "and write them to this JSON file")
    parser.add_argument("--step-only", action="store_true",
                        help="run warm-up and the timed steps only (launch-list captures)")
    parser.add_argument("--repeat-child", action="store_true", help=argparse.SUPPRESS)
    parser.add_argument("--reference-child", action="store_true", help=argparse.SUPPRESS)
    parser.add_argument("--profile", choices=["fused", "rms", "qkkv", "qk", "qkcache", "quant", "fp4",
                                              "projection"],
                        help="launch one operator at one shape and exit (ncu driver)")
    parser.add_argument("--tokens", type=int, default=1024)
    parser.add_argument("--hidden", type=int, default=4096)
    parser.add_argument("--heads", default="32,8")
    parser.add_argument("--dtype", default="bf16", choices=["bf16", "fp16", "fp32"])
    parser.add_argument("--version", type=int, default=0)
    parser.add_argument("--launches", type=int, default=5)
    parser.add_argument("--warm", action="store_true",
                        help="with --profile: no L2 flush between launches")
    args = parser.parse_args()
    if args.profile:
        profile_case(args)
        return
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")
    if args.repeat_child:
        repeat_child(args)
        return
    if args.reference_child:
        reference_child(args)
        return

    dist = Dist()
    if args.gpus > 1 and dist.world == 1:
        # not under torchrun: relaunch one process per GPU
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={args.gpus}", "--master-addr=127.0.0.1",
               "--master-port=29517", *sys.argv]
        raise SystemExit(subprocess.call(cmd))
    if dist.world > 1 and args.gpus != dist.world:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {dist.world}; using WORLD_SIZE",
              file=sys.stderr)

    if args.impl == "reference":
        if dist.rank != 0:
            return
        print(json.dumps(reference_arm(args)))
        return

    dist.init()
    try:
        line = gpu_arm(args, dist)
        if dist.rank == 0 and dist.world == 1 and not args.skip_cpu and not args.step_only:
            threads = host_threads()
            gbs, calls, elapsed, _ = cpu_port_timing(HEADLINE_ROWS, threads, None,
                                                     args.cpu_seconds)
            line["cpu_baseline"] = {
                "value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                "sample": f"{calls} in-place calls on the full [65536, 8192] bf16 x and residual "
                          f"in {elapsed:.1f} s (C restatement of the reference's PyTorch oracle, "
                          "OpenMP)"}
            line["roofline"] = line.pop("roofline")
        if dist.rank == 0:
            print(json.dumps(line))
    finally:
        dist.close()


if __name__ == "__main__":
    main()
