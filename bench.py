"""Multi-LoRA shrink+expand benchmark (BASELINE.json metric) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 1|2|3] [--path fused|rows]

Default workload (the headline): one decode batch of 256
tokens at Llama-3-8B projection shapes with 128 resident rank-16 adapters, adapter
ids Zipf(1.1); the three projections fused QKV (4096 -> 4096/1024/1024), gate/up
(4096 -> 2 x 14336) and down (14336 -> 4096).  x ~ N(0,1), A ~ N(0,1/K),
B ~ N(0,1/r), scale 2.0, all BF16, seeded synthetic data.  Config 2 (512 tokens,
256 retained-rank adapters, ranks U{4,8,16,32,64}, compact B, rsLoRA scales) and
config 3 (8192-token prefill in 32 geometric segments, 64 rank-64 adapters, 5120)
use the same harness.  One step = device grouping of the batch by adapter + shrink
+ expand of every projection.

``value``   tokens/s of the step replayed as a CUDA graph with inputs resident in
            HBM; L2 is flushed (a write larger than L2) before every timed step and
            the flush is outside the per-step CUDA events.
``e2e``     the same step through the public Python API with pinned host buffers:
            H2D of the step's activations and routing, D2H of the three outputs.
``roofline`` the dominant kernel's algorithmic bytes / its mean event time, against
            the measured HBM copy bandwidth in MEASURED_PEAKS.json.
``cpu_baseline`` the FP32 einsum over per-adapter gathers (the oracle port) on the
            host cores, on a bounded sample of steps (rank 0, N=1 only).

With N>1 (torchrun) every rank runs an independent replica of the workload
(replicas only: config 1 has no cross-GPU exchange); value = all ranks' tokens /
max over ranks of the device time.  ``--impl reference`` times the CPU oracle port
on the same workload (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "multi-LoRA shrink+expand tokens/s"

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the dominant
# call, from one ncu capture per (config, path, call); see profiles/ for the commands.
TRAFFIC = {
    (1, "fused", "gate_up_proj.fused"): (19.430144 + 75.358720 + 3.842816) * 1e6,
    (2, "fused", "proj.fused"): (51.121664 + 0.143360 + 49.703424 + 0.023040) * 1e6,
}


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=300)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", type=int, choices=sorted(CONFIGS), default=1)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--path", choices=("fused", "rows"), default="fused")
    p.add_argument("--allreduce", choices=("peer", "nccl"), default="peer",
                   help="tensor-parallel z sum: one kernel over NVLink peer memory, or NCCL")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--profile", action="store_true", help="short run for ncu (no sampling/baselines)")
    return p.parse_args()


# ----------------------------------------------------------------------------- workloads
def zipf_slots(rng, tokens, slots, s):
    ranks = np.arange(1, slots + 1, dtype=np.float64)
    p = ranks**-s
    return rng.choice(slots, size=tokens, p=p / p.sum()).astype(np.int32)


def geometric_segments(rng, tokens, segments, mean):
    """Contiguous segment lengths: geometric (mean `mean`, min 1), rescaled to sum `tokens`."""
    lengths = rng.geometric(1.0 / mean, size=segments).astype(np.float64)
    lengths = np.maximum(1, np.floor(lengths * tokens / lengths.sum())).astype(np.int64)
    lengths[np.argmax(lengths)] += tokens - lengths.sum()
    return lengths


def next_pow2(r):
    return 1 << (max(1, int(r)) - 1).bit_length()


# BASELINE.json configs (shapes and distributions); config 1 is the headline.
CONFIGS = {
    1: dict(
        workload="config1: decode BGMV, Llama-3-8B qkv/gate_up/down, 256 tokens, 128 adapters "
        "r=16, Zipf(1.1)",
        tokens=256, slots=128, cap=16,
        projections=(("qkv_proj", 4096, (4096, 1024, 1024)),
                     ("gate_up_proj", 4096, (14336, 14336)),
                     ("down_proj", 14336, (4096,))),
    ),
    2: dict(
        workload="config2: retained-rank decode, 512 tokens, 256 adapters, ranks U{4..64}, "
        "compact B, rsLoRA alpha=16, 4096->4096",
        tokens=512, slots=256, cap=64, projections=(("proj", 4096, (4096,)),),
    ),
    3: dict(
        workload="config3: prefill SGMV, 8192 tokens in 32 geometric segments (mean 256), "
        "64 adapters r=64, 5120->5120",
        tokens=8192, slots=64, cap=64, projections=(("proj", 5120, (5120,)),), prefill=True,
    ),
    4: dict(
        workload="config4: tensor-parallel decode, hidden 5120, intermediate 27648, 512 tokens, "
        "1024 adapters r=32, Zipf(1.0); gate/up column-parallel, down row-parallel with an "
        "all-reduce of the FP32 z rows",
        tokens=512, slots=1024, cap=32, hidden=5120, inter=27648, sharded=True,
    ),
}


def config_projections(config, world):
    """(name, in_dim, slice widths) of each projection on one rank of `world`."""
    c = CONFIGS[config]
    if not c.get("sharded"):
        return c["projections"]
    h, f = c["hidden"], c["inter"]
    if f % world or h % world:
        raise SystemExit(f"config {config} needs a rank count dividing {f} and {h}")
    # gate/up: full input, this rank's columns of both slices; down: this rank's input
    # columns and output columns.
    return (("gate_up_proj", h, (f // world, f // world)), ("down_proj", f // world, (h // world,)))


def config_routing(config, rng):
    """Per-slot ranks, scales and the token -> slot routing of a config."""
    c = CONFIGS[config]
    T, G = c["tokens"], c["slots"]
    if config == 1:
        ranks = np.full(G, 16)
        scales = np.full(G, 2.0)
        slots = zipf_slots(rng, T, G, 1.1)
    elif config == 4:
        ranks = np.full(G, 32)
        scales = np.full(G, 2.0)
        slots = zipf_slots(rng, T, G, 1.0)
    elif config == 2:
        ranks = rng.choice([4, 8, 16, 32, 64], size=G)
        scales = 16.0 / np.sqrt(ranks)
        slots = rng.integers(0, G, size=T).astype(np.int32)
    else:
        ranks = np.full(G, 64)
        scales = np.full(G, 2.0)
        lengths = geometric_segments(rng, T, 32, 256)
        owners = rng.integers(0, G, size=len(lengths))
        slots = np.repeat(owners, lengths).astype(np.int32)
    return ranks.astype(np.int32), scales.astype(np.float32), slots


class Projection:
    """One LoRA-augmented projection: packed A, compact B store, per-slot metadata."""

    def __init__(self, name, k, widths, ranks, scales, cap, tokens, device, gen, prefill=False):
        import torch

        from loraforge_b200.ops.fused import prefill_workspace_floats, workspace_floats

        self.name, self.K, self.widths = name, k, widths
        self.S, self.N = len(widths), sum(widths)
        self.cap, self.ranks_np, self.scales_np = cap, ranks, scales
        G, S, N, K = len(ranks), self.S, self.N, k
        self.a = (torch.randn(G, S * cap, K, generator=gen, device=device) / K**0.5).bfloat16()
        buckets = np.array([next_pow2(r) for r in ranks])
        offsets = np.concatenate(([0], np.cumsum(N * buckets)[:-1]))  # multiples of 8
        self.b = torch.randn(int(N * buckets.sum()), generator=gen, device=device).bfloat16()
        for g in range(G):  # B ~ N(0, 1/r), zero beyond the slot's rank
            view = self.b[offsets[g] : offsets[g] + N * buckets[g]].view(N, int(buckets[g]))
            view.mul_(1.0 / float(ranks[g]) ** 0.5)
            view[:, int(ranks[g]) :] = 0
        self.offsets_np, self.buckets_np = offsets, buckets
        self.b_offsets = torch.tensor(offsets, dtype=torch.int64, device=device)
        self.b_strides = torch.tensor(buckets, dtype=torch.int32, device=device)
        self.ranks = torch.tensor(ranks, dtype=torch.int32, device=device)
        self.scales = torch.tensor(scales, dtype=torch.float32, device=device)
        self.slice_offsets = torch.tensor(np.cumsum((0, *widths)), dtype=torch.int32, device=device)
        self.z = torch.zeros(tokens, S * cap, dtype=torch.bfloat16, device=device)
        sizer = prefill_workspace_floats if prefill else workspace_floats
        self.workspace = torch.zeros(sizer(tokens, K, S, cap), dtype=torch.float32, device=device)
        self.y = torch.zeros(tokens, N, dtype=torch.bfloat16, device=device)

    def b_rows(self, g):
        """Host copy of slot g's B rows [N, bucket] (for the CPU oracle)."""
        off, bucket = int(self.offsets_np[g]), int(self.buckets_np[g])
        return self.b_host[off : off + self.N * bucket].view(self.N, bucket)

    # Algorithmic bytes (the rank-r intermediate's round trip is not counted).
    def shrink_bytes(self, touched, t_active):
        return t_active * self.K * 2 + int(self.ranks_np[touched].sum()) * self.S * self.K * 2

    def expand_bytes(self, touched, t_active):
        return int(self.buckets_np[touched].sum()) * self.N * 2 + t_active * self.N * 2 * 2

    def flops(self, slots):
        r = self.ranks_np[slots[slots >= 0]]
        return int((2 * r * (self.S * self.K + self.N)).sum())


class Workload:
    def __init__(self, config, device, seed, world=1):
        import torch

        from loraforge_b200.ops.grouping import empty_routing

        c = CONFIGS[config]
        gen = torch.Generator(device=device).manual_seed(seed)
        rng = np.random.default_rng(seed)
        self.config, self.device, self.T, self.nslots = config, device, c["tokens"], c["slots"]
        self.prefill = c.get("prefill", False)
        self.sharded, self.world = c.get("sharded", False), world
        projections = config_projections(config, world)
        self.ranks_np, self.scales_np, self.slots_np = config_routing(config, rng)
        self.slots = torch.from_numpy(self.slots_np).to(device)
        self.x = {}
        for _, k, _ in projections:
            if k not in self.x:
                self.x[k] = torch.randn(self.T, k, generator=gen, device=device).bfloat16()
        self.projections = [
            Projection(n, k, w, self.ranks_np, self.scales_np, c["cap"], self.T, device, gen,
                       c.get("prefill", False))
            for n, k, w in projections
        ]
        self.routing = empty_routing(self.T, device)
        self.touched = np.unique(self.slots_np[self.slots_np >= 0])
        self.t_active = int((self.slots_np >= 0).sum())

    def x_of(self, p):
        return self.x[p.K]

    def bytes_per_step(self):
        return sum(
            p.shrink_bytes(self.touched, self.t_active) + p.expand_bytes(self.touched, self.t_active)
            for p in self.projections
        ) + self.T * 4

    def flops_per_step(self):
        return sum(p.flops(self.slots_np) for p in self.projections)


def run_step(w, mark=None):
    """Grouping + LoRA shrink/expand of every projection through the public API.

    ``w.path == "fused"``: lora_shrink_expand per projection (prefill configs:
    lora_shrink_expand_prefill over segments of up to 128 tokens on the tcgen05 tiles);
    ``"rows"``: row_shrink + row_expand per projection (the reference's operator pair);
    tensor-parallel configs: gate/up column-parallel, down as shrink, all-reduce of the
    z rows over the ranks, expand.  ``mark(label)``, when given, records a CUDA event
    that starts the interval named `label` (ended by the next mark or "end").
    """
    from loraforge_b200.ops import row_expand, row_shrink
    from loraforge_b200.ops.fused import (
        lora_shrink_expand,
        lora_shrink_expand_prefill,
        sgmv_expand,
        sgmv_shrink,
        z_rows,
    )
    from loraforge_b200.ops.grouping import group_tokens

    mark = mark or (lambda label: None)
    prefill = w.prefill and w.path == "fused"
    fused_op = lora_shrink_expand_prefill if prefill else lora_shrink_expand
    r = group_tokens(w.slots, w.nslots, chunk=128 if prefill else 16, runs=prefill, out=w.routing)
    routing = dict(
        segment_indptr=r.segment_indptr, segment_slots=r.segment_slots,
        token_indices=r.token_indices, segment_count=r.segment_count,
    )
    for p in w.projections:
        meta = dict(b_offsets=p.b_offsets, b_strides=p.b_strides, ranks=p.ranks,
                    scales=p.scales, slice_offsets=p.slice_offsets, **routing)
        x = w.x_of(p)
        if w.sharded and p.name == "down_proj":
            mark(f"{p.name}.shrink")
            sgmv_shrink(x, p.a, p.b, p.y, workspace=p.workspace, **meta, num_slices=p.S)
            if w.world > 1:
                import torch.distributed as dist

                mark(f"{p.name}.allreduce")
                z = z_rows(p.workspace, w.T, p.K, p.S, p.cap)
                if getattr(w, "peer", None) is not None:
                    w.peer(z)
                else:
                    dist.all_reduce(z)
            mark(f"{p.name}.expand")
            sgmv_expand(x, p.a, p.b, p.y, workspace=p.workspace, **meta, num_slices=p.S)
        elif w.path == "fused":
            mark(f"{p.name}.fused")
            fused_op(x, p.a, p.b, p.y, **meta, num_slices=p.S, workspace=p.workspace)
        else:
            mark(f"{p.name}.shrink")
            row_shrink(x, p.a, p.z, w.slots, p.ranks, num_slices=p.S, max_rank=p.cap)
            mark(f"{p.name}.expand")
            row_expand(p.z, p.b, p.y, **meta)
    mark("end")


def launches_per_step(w):
    # grouping + two kernels per projection (shrink and expand; the prefill pair too)
    return 1 + 2 * len(w.projections)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """NVML SM-clock / throttle-reason sampling during the timed region (read-only)."""

    REASONS = {
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self._nvml = pynvml
            uuid = getattr(torch.cuda.get_device_properties(index), "uuid", None)
            if uuid is not None:
                self._h = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{uuid}")
            else:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._reasons_fn = getattr(
                pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None
            ) or getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
        except Exception:  # NVML unavailable: report no clock record
            self._nvml = None

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = self._reasons_fn(self._h)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def record(self):
        if not self.samples:
            return None
        return {
            "sm_mhz": statistics.median(self.samples),
            "sm_max_mhz": self.max_mhz,
            "samples": len(self.samples),
            "reasons": sorted(self.reasons),
        }


# ----------------------------------------------------------------------------- timing
def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def time_graph(w, steps, warmup, flush):
    """Replay the captured step `steps` times; per-step and per-kernel CUDA events."""
    import torch

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            run_step(w)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run_step(w)
    for _ in range(warmup):
        flush.zero_()
        graph.replay()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        starts[i].record()
        graph.replay()
        ends[i].record()
    torch.cuda.synchronize()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    del graph
    # Kernel breakdown: eager launches queued behind a device sleep so that host
    # launch latency never shows up between the events; L2 flushed before each step.
    per_kernel = {}
    for _ in range(min(steps, 50)):
        marks = []

        def mark(label):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            marks.append((label, e))

        flush.zero_()
        torch.cuda._sleep(4_000_000)
        run_step(w, mark=mark)
        torch.cuda.synchronize()
        for (label, e0), (_, e1) in zip(marks, marks[1:]):
            per_kernel.setdefault(label, []).append(e0.elapsed_time(e1))
    return step_ms, {k: statistics.mean(v) for k, v in per_kernel.items()}


def time_e2e(w, steps, warmup):
    """Public API with host buffers: H2D inputs, the step, D2H outputs, per step."""
    import torch

    host_x = {k: v.cpu().pin_memory() for k, v in w.x.items()}
    host_slots = w.slots.cpu().pin_memory()
    host_out = [torch.empty(p.y.shape, dtype=p.y.dtype).pin_memory() for p in w.projections]
    h2d = sum(t.numel() * 2 for t in host_x.values()) + host_slots.numel() * 4
    d2h = sum(t.numel() * 2 for t in host_out)

    def one():
        for k, t in host_x.items():
            w.x[k].copy_(t, non_blocking=True)
        w.slots.copy_(host_slots, non_blocking=True)
        run_step(w)
        for p, h in zip(w.projections, host_out):
            h.copy_(p.y, non_blocking=True)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        one()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps, h2d, d2h


def cpu_baseline(w, budget_s=15.0):
    """FP32 einsum over per-adapter gathers on the host (oracle port), bounded sample."""
    import torch

    from oracle.cpu_reference import lora_delta_fp32

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    slots = w.slots_np
    xs = {k: v.float().cpu() for k, v in w.x.items()}
    hosts = []
    for p in w.projections:
        p.b_host = p.b.cpu()
        hosts.append((p, p.a.cpu(), p.slice_offsets.cpu().numpy()))

    def step():
        for p, a_host, bounds in hosts:
            lora_delta_fp32(xs[p.K], a_host, p.b_rows, slots, w.ranks_np, w.scales_np, bounds)

    t0 = time.perf_counter()
    step()  # warm-up (also sizes the sample)
    first = time.perf_counter() - t0
    times = []
    begin = time.perf_counter()
    while time.perf_counter() - begin < budget_s and len(times) < 50:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if first > budget_s:
            break
    per_step = statistics.median(times)
    return {
        "value": w.T / per_step,
        "unit": "tokens/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{len(times)} full steps ({len(w.projections)} projections x {w.T} tokens), "
        "median",
    }


# ----------------------------------------------------------------------------- main
def init_distributed():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def main():
    args = parse_args()
    import torch

    c = CONFIGS[args.config]
    config = {
        "workload": c["workload"],
        "tokens": c["tokens"],
        "adapters": c["slots"],
        "rank_capacity": c["cap"],
        "l2": "flushed before every timed step (256 MiB write, outside the step events)",
    }
    if args.impl == "reference":
        return main_reference(args, config)
    world, rank, local = init_distributed()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    w = Workload(args.config, device, args.seed + rank, world)
    w.path = args.path
    w.peer = None
    if w.sharded and world > 1 and args.allreduce == "peer":
        from loraforge_b200.ops.fused import z_rows
        from loraforge_b200.ops.sharded import PeerAllReduce

        down = next(p for p in w.projections if p.name == "down_proj")
        w.peer = PeerAllReduce(z_rows(down.workspace, w.T, down.K, down.S, down.cap).numel(), device=device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    steps, warmup = args.steps, max(3, args.warmup)
    barrier(world)
    with ClockSampler(local) as clocks:
        step_ms, per_kernel = time_graph(w, steps, warmup, flush)
    barrier(world)
    total_ms = max_over_ranks(sum(step_ms), world)
    ms_per_step = total_ms / steps
    # Replicas: every rank processes its own batch; tensor-parallel: the ranks share one.
    value = (1 if w.sharded else world) * w.T * steps / (total_ms / 1e3)
    peak, peak_kind = measured_peaks()
    kernels = {k: v for k, v in per_kernel.items() if k.split(".")[1] in ("shrink", "expand", "fused")}
    dominant = max(kernels, key=kernels.get)
    name, kind = dominant.split(".")
    p = next(p for p in w.projections if p.name == name)
    alg = {
        "shrink": p.shrink_bytes(w.touched, w.t_active),
        "expand": p.expand_bytes(w.touched, w.t_active),
        "fused": p.shrink_bytes(w.touched, w.t_active) + p.expand_bytes(w.touched, w.t_active),
    }[kind]
    achieved = alg / (per_kernel[dominant] * 1e-3) / 1e9
    result = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "strong" if w.sharded else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": f"synthetic (seeded; BASELINE config {args.config} shapes and distributions)",
        "config": config | {"parallelism": f"tp{world}" if w.sharded else f"replicas{world}",
                            "path": w.path}
                  | ({"z_allreduce": args.allreduce} if w.sharded and world > 1 else {}),
        "hbm_gbs_step": w.bytes_per_step() / (ms_per_step * 1e-3) / 1e9,
        "bytes_per_step": w.bytes_per_step(),
        "flops_per_step": w.flops_per_step(),
        "kernel_ms": per_kernel,
        "roofline": {
            "bound": "hbm",
            "kernel": dominant,
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
            "traffic": TRAFFIC.get((args.config, w.path, dominant)),
        },
        "gpu_launches": launches_per_step(w) * steps,
        "clocks": clocks.record(),
    }
    if not args.no_e2e and not args.profile:
        e2e_ms, h2d, d2h = time_e2e(w, max(10, steps // 10), 3)
        e2e_ms = max_over_ranks(e2e_ms, world)
        result["e2e"] = {
            "value": world * w.T / (e2e_ms * 1e-3),
            "unit": "tokens/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
        }
    if "down_proj.allreduce" in per_kernel:  # the z all-reduce, timed on its own
        result["allreduce_us"] = max_over_ranks(per_kernel["down_proj.allreduce"], world) * 1e3
    if rank == 0 and world == 1 and not w.sharded and not args.no_cpu_baseline and not args.profile:
        result["cpu_baseline"] = cpu_baseline(w)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if w.peer is not None:
        w.peer.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main_reference(args, config):
    """CPU oracle port of the reference path on the host cores (rank 0 only)."""
    import torch

    if int(os.environ.get("RANK", "0")) != 0:
        return
    w = Workload(args.config, torch.device("cpu"), args.seed)
    budget = max(10.0, min(120.0, 2.0 * (args.steps + args.warmup)))
    base = cpu_baseline(w, budget_s=budget)
    print(
        json.dumps(
            {
                "impl": "reference",
                "metric": METRIC,
                "value": base["value"],
                "unit": "tokens/s",
                "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
                "steps": args.steps,
                "warmup": args.warmup,
                "ms_per_step": 1e3 * w.T / base["value"],
                "higher_is_better": True,
                "scaling": "weak",
                "vs_baseline": None,
                "dtype": "f32",
                "data": f"synthetic (seeded; BASELINE config {args.config} shapes and distributions)",
                "config": config | {"parallelism": "host cores"},
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "tokens/s",
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            }
        ),
        flush=True,
    )


if __name__ == "__main__":
    main()
