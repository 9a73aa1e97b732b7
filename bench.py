"""Benchmark: achieved HBM GB/s (% of B200 peak) and us/call of the fused
normalisation path, at 1..8 GPUs.

Workload (one "step"): the in-place residual-add + RMSNorm sweep the metric is
quoted on -- tokens in {1, 4, 16, 64, 256, 1024} x hidden in {768, 1024, 2048,
4096} x {bf16, fp16}, x and residual ~ N(0, 1), weight ~ N(1, 0.1), eps 1e-6:
48 calls of ``fused_add_rms_norm_inplace``, replayed as one CUDA graph. L2 is
flushed (a 512 MiB write) before every timed step, outside the timed events.
``value`` = algorithmic bytes of all ranks' steps / max-over-ranks device time.

Also reported on the same line:
  * ``roofline`` -- the dominant kernel of the step (the longest call), its
    algorithmic bytes per launch over its launch duration, against the
    measured HBM copy peak. Launch durations (``per_shape``) come from CUDA
    events around a graph of R back-to-back calls of one shape on R distinct
    buffer sets (every call reads data that is not in L2), replayed after an
    L2 flush: duration = replay time / R;
  * ``e2e`` -- the same sweep through the public API with the inputs copied
    from pinned host memory and both outputs copied back inside the timed
    region (one packed upload and one download per step, consecutive steps
    overlapping on two device buffer sets);
  * ``per_op`` -- us/call and GB/s of every operator at the other workload
    shapes (batch-1 and wide-batch decode Q/K norm + RoPE + KV store, the
    prefill fused add [65536, 8192] and Q/K prefill of 32768 tokens, and the
    fp32 RMSNorm rows), timed the same way as ``per_shape``;
  * ``cpu_baseline`` -- the C oracle on the host cores (rank 0, N=1 only).

``--impl reference`` times the reference path's CPU implementation (the C
restatement of its PyTorch oracle) on the host cores instead.

Multi-GPU: launched one process per GPU by torchrun; each rank runs the same
per-rank workload on its own GPU (rows / sequences sharded, no collective on
the data path). NCCL is used only for the barrier and the max-over-ranks time.
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


def sweep_shapes():
    return [(t, h, name) for name in DTYPES for t in TOKENS for h in HIDDEN]


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
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
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


def dram_traffic_per_launch():
    """dram bytes read + written per launch of the dominant kernel, from the
    committed ncu summary (profiles/dram_traffic.txt), or None."""
    path = ROOT / "profiles" / "dram_traffic.txt"
    if not path.exists():
        return None
    out = {}
    for line in path.read_text().splitlines():
        if "=" in line and not line.startswith("#"):
            k, v = line.split("=", 1)
            out[k.strip()] = v.strip()
    return out


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
# GPU arm
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
    loading stays out of it)."""
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


class SweepData:
    def __init__(self, seed: int):
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.items = []
        for t, h, name in sweep_shapes():
            dt = DTYPES[name]
            x = torch.randn(t, h, device="cuda", generator=g).to(dt)
            r = torch.randn(t, h, device="cuda", generator=g).to(dt)
            w = (1.0 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(dt)
            self.items.append((t, h, name, x, r, w))
        self.bytes = sum(fused_bytes(t, h, x.element_size()) for t, h, _, x, _, _ in self.items)

    def run(self, ops):
        for _, _, _, x, r, w in self.items:
            ops.fused_add_rms_norm_inplace(x, r, w, EPS)


def per_shape_times(ops, data: "SweepData", flush: "Flusher", dist: "Dist", args) -> list:
    """Per-launch duration of every sweep shape: a graph of R back-to-back calls
    on R distinct buffer sets (every call reads data that is not in L2),
    replayed after an L2 flush; duration = replay time / R."""
    per_shape = []
    g = torch.Generator(device="cuda").manual_seed(77 + dist.rank)
    for t, h, name, x, r, w in data.items:
        nbytes = fused_bytes(t, h, x.element_size())
        sets = max(1, min(64, (256 << 20) // nbytes))
        bufs = [(x, r)] + [(torch.randn(t, h, device="cuda", generator=g).to(x.dtype),
                            torch.randn(t, h, device="cuda", generator=g).to(x.dtype))
                           for _ in range(sets - 1)]
        calls = [(lambda bx=bx, br=br, w=w: ops.fused_add_rms_norm_inplace(bx, br, w, EPS))
                 for bx, br in bufs]
        shape_graph, _ = capture(calls)
        us = time_graph(shape_graph, flush, max(3, args.reps)) / sets
        del shape_graph, bufs, calls
        per_shape.append({"tokens": t, "hidden": h, "dtype": name, "us": round(dist.max(us), 3),
                          "bytes": nbytes, "calls_per_graph": sets})
    for p in per_shape:
        p["gbs"] = round(p["bytes"] / (p["us"] * 1e-6) / 1e9, 1)
    return per_shape


def sweep_step_ms(ops, data: "SweepData", flush: "Flusher", steps: int, warmup: int,
                  dist: "Dist") -> float:
    """Mean device time of one step (the 48-call sweep as one CUDA graph), L2
    flushed before every step outside the timed events."""
    graph, _ = capture([lambda: data.run(ops)])
    for _ in range(warmup):
        flush()
        graph.replay()
    dist.barrier()
    pairs = []
    for _ in range(steps):
        flush()
        a, b = event_pair()
        a.record()
        graph.replay()
        b.record()
        pairs.append((a, b))
    dist.barrier()
    return sum(a.elapsed_time(b) for a, b in pairs) / steps


def gpu_arm(args, dist: Dist) -> dict:
    import sm120_rmsnorm as ops

    dev = torch.device("cuda", torch.cuda.current_device())
    flush = Flusher()
    data = SweepData(seed=1234 + dist.rank)

    launches_per_step = len(data.items)
    clocks = ClockSampler(sampled_gpus(dist.world) if dist.rank == 0 else None)
    clocks.__enter__()
    try:
        step_ms = sweep_step_ms(ops, data, flush, args.steps, args.warmup, dist)
        if args.step_only:  # the timed steps alone (for a launch-list capture)
            return {"metric": "step only", "ms_per_step": round(dist.max(step_ms), 5),
                    "gpu_launches": launches_per_step * args.steps}
        line = _measure_rest(args, dist, ops, flush, data, step_ms, launches_per_step)
    finally:
        clocks.__exit__(None, None, None)
    line["clocks"] = clocks.summary() if dist.rank == 0 else None
    return line


def _measure_rest(args, dist, ops, flush, data, step_ms, launches_per_step) -> dict:
    dev = torch.device("cuda", torch.cuda.current_device())
    step_ms_max = dist.max(step_ms)
    value = data.bytes * dist.world / (step_ms_max * 1e-3) / 1e9

    per_shape = per_shape_times(ops, data, flush, dist, args)
    for p in per_shape:
        p["gbs"] = round(p["bytes"] / (p["us"] * 1e-6) / 1e9, 1)
    dominant = max(per_shape, key=lambda p: p["us"])
    peak, peak_source = measured_hbm_peak()
    traffic = dram_traffic_per_launch()
    traffic_value = None
    if traffic and traffic.get("config") == \
            f"fused_add_rms_norm_inplace {dominant['tokens']}x{dominant['hidden']}":
        traffic_value = int(float(traffic.get("dram_bytes_per_launch", "nan")))
    roofline = {"bound": "hbm", "achieved": dominant["gbs"], "peak": peak, "unit": "GB/s",
                "frac": round(dominant["gbs"] / peak, 4), "traffic": traffic_value,
                "kernel": f"fused_add_rms_norm_inplace {dominant['dtype']} "
                          f"{dominant['tokens']}x{dominant['hidden']}",
                "timing": "CUDA events around a graph of R back-to-back calls of this "
                          "shape on R distinct buffer sets, replayed after an L2 flush; "
                          "duration = replay time / R",
                "algorithmic_bytes_per_launch": dominant["bytes"],
                "launch_us": dominant["us"], "peak_source": peak_source + ", of measured"
                if peak_source.startswith("measured") else peak_source + ", of fallback"}

    # end to end through the public API with pinned host buffers. Every step
    # uploads the step's inputs (each call's x and r, packed 256-byte aligned
    # in one pinned host buffer) in one copy, runs the 48 calls on views of
    # the device copy and downloads the results in one copy. Consecutive steps
    # rotate over three device buffer sets, so step k + 1's upload runs while
    # step k computes and downloads and no upload waits for a compute
    # (uploads, calls and downloads on three streams; both PCIe directions
    # busy), as a streaming engine would.
    # E steps are captured as one CUDA graph and the graph is timed; per-step
    # time = elapsed / E.
    offsets, total = [], 0
    for _, _, _, x, r, _ in data.items:
        nb = x.numel() * x.element_size()
        offsets.append((total, total + ((nb + 255) // 256) * 256, nb))
        total += 2 * ((nb + 255) // 256) * 256
    host_in = torch.empty(total, dtype=torch.uint8).pin_memory()
    host_out = torch.empty(total, dtype=torch.uint8).pin_memory()
    for (ox, orr, nb), (_, _, _, x, r, _) in zip(offsets, data.items):
        host_in[ox:ox + nb].copy_(x.reshape(-1).view(torch.uint8).cpu())
        host_in[orr:orr + nb].copy_(r.reshape(-1).view(torch.uint8).cpu())
    dev_sets = [torch.empty(total, dtype=torch.uint8, device="cuda") for _ in range(3)]

    def views(buf):
        out = []
        for (ox, orr, nb), (t, h, _, x, _, w) in zip(offsets, data.items):
            out.append((buf[ox:ox + nb].view(x.dtype).view(t, h),
                        buf[orr:orr + nb].view(x.dtype).view(t, h), w))
        return out

    set_views = [views(b) for b in dev_sets]
    h2d = total
    up, compute, down = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()

    def e2e_steps_run(n_steps):
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
                for x, r, w in set_views[i]:
                    ops.fused_add_rms_norm_inplace(x, r, w, EPS)
                computed = torch.cuda.Event()
                computed.record(compute)
            down.wait_event(computed)
            with torch.cuda.stream(down):
                host_out.copy_(dev_sets[i], non_blocking=True)
                freed[i] = torch.cuda.Event()
                freed[i].record(down)
        for stream in (up, compute, down):
            origin.wait_stream(stream)

    e2e_steps = max(6, args.steps // 5)
    e2e_steps_run(3)  # eager once, then capture
    torch.cuda.synchronize()
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_steps_run(e2e_steps)
    for _ in range(max(1, args.warmup // 2)):
        e2e_graph.replay()
    dist.barrier()
    a, b = event_pair()
    a.record()
    e2e_graph.replay()
    b.record()
    b.synchronize()
    e2e_ms = dist.max(a.elapsed_time(b) / e2e_steps)
    e2e = {"value": round(data.bytes * dist.world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
           "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d * dist.world,
           "d2h_bytes_per_step": h2d * dist.world,
           "path": "sm120_rmsnorm.fused_add_rms_norm_inplace on views of one packed device "
                   "buffer per step: one pinned-host upload and one download per step, three "
                   "device buffer sets in rotation so that a step's upload overlaps the "
                   "previous step's calls and download (three streams), "
                   f"{e2e_steps} steps per CUDA graph"}

    per_op = {} if args.skip_per_op else per_op_suite(ops, flush, dist, args)
    extensions = {} if args.skip_per_op else extension_suite(flush, dist, args)
    engine = {} if args.skip_per_op else engine_suite(flush, dist, args)
    projection = {} if args.skip_per_op else projection_suite(flush, dist, args)

    return {
        "metric": "achieved HBM GB/s (% of B200 peak) and us/call per op at 1/2/4/8 GPUs",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms_max, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16+fp16 (fp32 accumulate)",
        "data": "synthetic (seeded N(0,1) activations, N(1,0.1) weights)",
        "config": {"workload": "in-place residual add + RMSNorm sweep: tokens "
                               "{1,4,16,64,256,1024} x hidden {768,1024,2048,4096} x "
                               "{bf16,fp16}, one CUDA graph of 48 launches per step",
                   "global_batch": len(data.items) * dist.world,
                   "bytes_per_step_per_gpu": data.bytes, "parallelism": f"dp{dist.world}"
                   f" (each rank its own rows, no collective)",
                   "l2": "flushed (512 MiB write) before every timed step and every "
                         "per-launch timing, outside the events"},
        "roofline": roofline, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
        "per_shape": per_shape, "per_op": per_op, "extensions": extensions, "engine": engine,
        "projection": projection,
        "device": torch.cuda.get_device_name(dev),
    }


def per_op_suite(ops, flush: Flusher, dist: Dist, args) -> dict:
    """us/call and GB/s of each operator at the other workload shapes.

    Each entry is a CUDA graph of R back-to-back calls on R distinct buffer
    sets (R up to 64, fewer when a call moves more than 4 MiB), replayed after
    an L2 flush, so every call reads inputs that are not in L2; us/call is the
    replay time over R.
    """
    out = {}
    reps = max(3, args.reps)
    g = torch.Generator(device="cuda").manual_seed(99 + dist.rank)
    cpu_g = torch.Generator().manual_seed(7 + dist.rank)
    bf = torch.bfloat16

    def rope_cache(n):
        inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device="cuda") / 128))
        f = torch.outer(torch.arange(n, dtype=torch.float32, device="cuda"), inv)
        return torch.cat((f.cos(), f.sin()), dim=-1)

    cache = rope_cache(32768)

    def sets_for(nbytes):
        return max(1, min(64, (256 << 20) // max(nbytes, 1)))

    def record(name, calls, nbytes):
        graph, _ = capture(calls)
        us = dist.max(time_graph(graph, flush, reps) / len(calls))
        out[name] = {"us": round(us, 3), "bytes": nbytes,
                     "gbs": round(nbytes / (us * 1e-6) / 1e9, 1), "calls_per_graph": len(calls)}
        del graph

    # fp32 RMSNorm rows of 1024 (the CPU-runnable workload), on the GPU
    for t in (1, 4, 16, 64, 256):
        nbytes = rms_bytes(t, 1024, 4)
        calls = []
        for _ in range(sets_for(nbytes)):
            x = torch.randn(t, 1024, device="cuda", generator=g)
            w = 1.0 + 0.1 * torch.randn(1024, device="cuda", generator=g)
            y = torch.empty_like(x)
            calls.append(lambda x=x, w=w, y=y: ops.rms_norm_out(x, w, y, EPS))
        record(f"rms_norm fp32 {t}x1024", calls, nbytes)

    # Qwen3 decode Q/K norm + RoPE + paged KV store (one cache per case,
    # distinct slots and positions per buffer set)
    def qk_case(name, b, hq, hk, blocks, contiguous):
        nbytes = qk_kv_bytes(b, hq, hk, 2)
        n_sets = sets_for(nbytes)
        kc = torch.zeros(blocks, 16, hk, 128, device="cuda", dtype=bf)
        vc = torch.zeros_like(kc)
        qw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
        kw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(bf)
        all_slots = torch.randperm(blocks * 16, generator=cpu_g)[: b * n_sets].to(torch.int32)
        calls = []
        for i in range(n_sets):
            q = torch.randn(b, hq, 128, device="cuda", generator=g).to(bf)
            k = torch.randn(b, hk, 128, device="cuda", generator=g).to(bf)
            v = torch.randn(b, hk, 128, device="cuda", generator=g).to(bf)
            if contiguous:
                pos = torch.arange(b, device="cuda")
                slots = torch.arange(b, device="cuda", dtype=torch.int32)
            else:
                pos = torch.randperm(32768, generator=cpu_g)[:b].cuda()
                slots = all_slots[i * b:(i + 1) * b].cuda()
            calls.append(lambda q=q, k=k, v=v, pos=pos, slots=slots: ops.fused_qk_rms_norm_rope_kv(
                q, k, v, qw, kw, pos, cache, kc, vc, slots, EPS))
        record(name, calls, nbytes)

    qk_case("qk_kv decode bf16 B=1 16/8", 1, 16, 8, 2048, False)
    for b in (64, 256, 1024):
        qk_case(f"qk_kv decode bf16 B={b} 32/8", b, 32, 8, 65536, False)
    qk_case("qk_kv prefill bf16 32768 tokens 64/8", 32768, 64, 8, 2048, True)

    # prefill residual add + RMSNorm (4.3 GB per call: one call per graph)
    x = torch.randn(65536, 8192, device="cuda", generator=g).to(bf)
    r = torch.randn(65536, 8192, device="cuda", generator=g).to(bf)
    w = (1 + 0.1 * torch.randn(8192, device="cuda", generator=g)).to(bf)
    record("fused_add_rms_norm_inplace prefill bf16 65536x8192",
           [lambda: ops.fused_add_rms_norm_inplace(x, r, w, EPS)], fused_bytes(65536, 8192, 2))
    del x, r
    return out


def qk_cache_bytes(t: int, hq: int, hk: int, s: int, d: int = 128, rotary: int = 128,
                   cache_elem: int | None = None) -> int:
    # as qk_kv_bytes, with the two cache stores at the cache element size
    cache_elem = s if cache_elem is None else cache_elem
    return (t * (s * d * (2 * hq + 3 * hk) + 2 * cache_elem * d * hk + 8 + 4 + 4 * rotary)
            + 2 * d * s)


def norm_quant_bytes(t: int, h: int, s: int, add: bool, dynamic: bool) -> int:
    # x read (and r read + written), fp8 result written, weight once, scales
    return t * h * s * (3 if add else 1) + t * h + h * s + (4 * t if dynamic else 0)


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
        ours = DecodeGraph(layers, batch, cos_sin, kcs, vcs)
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


def cpu_sweep_gbs(seconds: float, threads: int, passes: int | None = None):
    from oracle import oracle

    oracle.build()
    oracle.set_threads(threads)
    g = torch.Generator().manual_seed(4321)
    items = []
    for t, h, name in sweep_shapes():
        dt = DTYPES[name]
        x = torch.randn(t, h, generator=g).to(dt)
        r = torch.randn(t, h, generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(h, generator=g)).to(dt)
        items.append((x, r, w))
    total = sum(fused_bytes(x.shape[0], x.shape[1], x.element_size()) for x, _, _ in items)
    for x, r, w in items:  # warm-up pass
        oracle.fused_add_rms_norm_out(x, r, w, x, r, EPS)
    done, t0 = 0, time.perf_counter()
    while True:
        for x, r, w in items:
            oracle.fused_add_rms_norm_out(x, r, w, x, r, EPS)
        done += 1
        elapsed = time.perf_counter() - t0
        if (passes is not None and done >= passes) or (passes is None and elapsed >= seconds):
            break
    return total * done / elapsed / 1e9, done, elapsed


class ReferenceKernels:
    """The reference project's own CUDA kernels (compiled for sm_100a from its
    sources by oracle/build_ref.py), called with its ops.py default versions."""

    def __init__(self, module):
        self.m = module

    def fused_add_rms_norm_inplace(self, x, r, w, eps=EPS, version=0):
        self.m.fused_add_rms_norm_inplace(x, r, w, eps, version)

    def rms_norm_out(self, x, w, out, eps=EPS, version=2):
        self.m.rms_norm_out(x, w, out, eps, version)

    def fused_qk_rms_norm_rope_kv(self, q, k, v, qw, kw, pos, cache, kc, vc, slots, eps=EPS,
                                  version=1):
        self.m.fused_qk_rms_norm_rope_kv(q, k, v, qw, kw, pos, cache, kc, vc, slots, eps, version)


def reference_kernels_gpu(args, dist: Dist) -> dict:
    """The reference's CUDA kernels on this B200, same workload and timing as
    the main arm (the SM120 kernels rebuilt for sm_100a: the bar to beat)."""
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    from oracle import build_ref

    module = build_ref.load()
    if module is None:
        return {"unavailable": "the reference's kernels were not built (oracle/build_ref.py "
                               "needs the reference checkout)"}
    torch.cuda.set_device(0)
    ops = ReferenceKernels(module)
    flush = Flusher()
    data = SweepData(seed=1234)
    step_ms = sweep_step_ms(ops, data, flush, args.steps, args.warmup, dist)
    per_shape = per_shape_times(ops, data, flush, dist, args)
    per_op = {} if args.skip_per_op else per_op_suite(ops, flush, dist, args)
    return {"value": round(data.bytes / (step_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(step_ms, 5),
            "build": "reference csrc/rmsnorm_kernels.cu + bindings.cpp, nvcc -O3 "
                     "--use_fast_math -gencode arch=compute_100a,code=sm_100a",
            "per_shape": per_shape, "per_op": per_op}


def pytorch_cpu_reference_gbs(steps: int, threads: int) -> dict:
    """The reference's PyTorch oracle math (residual add + RMSNorm,
    reference.py:14-24 in the reference project; restated op for op in
    sm120_rmsnorm/reference.py, loaded here by file path so nothing else of
    the package is imported) on the host CPU over the sweep."""
    import importlib.util

    path = ROOT / "sm120-norm-fusion-kernels_b200" / "sm120_rmsnorm" / "reference.py"
    spec = importlib.util.spec_from_file_location("sweep_reference_math", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(4321)
    items = []
    for t, h, name in sweep_shapes():
        dt = DTYPES[name]
        items.append((torch.randn(t, h, generator=g).to(dt), torch.randn(t, h, generator=g).to(dt),
                      (1 + 0.1 * torch.randn(h, generator=g)).to(dt)))
    total = sum(fused_bytes(x.shape[0], x.shape[1], x.element_size()) for x, _, _ in items)
    for x, r, w in items:
        module.fused_add_rms_norm_reference(x, r, w, EPS)
    t0 = time.perf_counter()
    for _ in range(steps):
        for x, r, w in items:
            module.fused_add_rms_norm_reference(x, r, w, EPS)
    elapsed = time.perf_counter() - t0
    return {"value": round(total * steps / elapsed / 1e9, 3), "unit": "GB/s", "threads": threads,
            "sample": f"{steps} passes over the 48-call sweep, {elapsed:.2f} s"}


def reference_arm(args, dist: Dist) -> dict:
    """The reference path's CPU implementation (C restatement of its PyTorch
    oracle) on the host cores, on the same sweep; rank 0 only."""
    threads = host_threads()
    from oracle import oracle

    oracle.build()
    oracle.set_threads(threads)
    for _ in range(args.warmup):
        cpu_sweep_gbs(0, threads, passes=1)
    gbs, passes, elapsed = cpu_sweep_gbs(0, threads, passes=args.steps)
    sample = (f"{passes} passes over the 48-call sweep (one step each), "
              f"{elapsed:.2f} s of CPU time")
    return {
        "impl": "reference",
        "metric": "achieved HBM GB/s (% of B200 peak) and us/call per op at 1/2/4/8 GPUs",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed / passes * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16+fp16 (fp32 accumulate)", "data": "synthetic",
        "config": {"workload": "in-place residual add + RMSNorm sweep: tokens "
                               "{1,4,16,64,256,1024} x hidden {768,1024,2048,4096} x "
                               "{bf16,fp16}", "parallelism": "host cores"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's CPU path is its PyTorch oracle (sm120_rmsnorm/reference.py), "
                "which cannot travel; this is its C restatement (oracle/norm_oracle.c), "
                "pinned to the reference's own outputs by the golden-vector tests",
        "reference_pytorch_cpu": pytorch_cpu_reference_gbs(max(3, args.steps // 4), threads),
        "reference_kernels_b200": reference_kernels_gpu(args, dist),
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
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--reps", type=int, default=10, help="launches per per-kernel timing")
    parser.add_argument("--impl", choices=["b200", "reference"], default="b200")
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--skip-per-op", action="store_true")
    parser.add_argument("--skip-cpu", action="store_true")
    parser.add_argument("--step-only", action="store_true",
                        help="run warm-up and the timed steps only (launch-list captures)")
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
        print(json.dumps(reference_arm(args, dist)))
        return

    dist.init()
    try:
        line = gpu_arm(args, dist)
        if dist.rank == 0 and dist.world == 1 and not args.skip_cpu and not args.step_only:
            threads = host_threads()
            gbs, passes, elapsed = cpu_sweep_gbs(args.cpu_seconds, threads)
            line["cpu_baseline"] = {
                "value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                "sample": f"{passes} passes over the 48-call sweep in {elapsed:.1f} s "
                          f"(C restatement of the reference's PyTorch oracle, OpenMP)"}
        if dist.rank == 0:
            print(json.dumps(line))
    finally:
        dist.close()


if __name__ == "__main__":
    main()
