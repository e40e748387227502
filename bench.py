"""Multi-LoRA shrink+expand benchmark (BASELINE.json metric) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 1|2|3|4] [--path fused|rows|bgmv|vllm|base_gemm|base_cublas] [--no-sub]

Default workload: BASELINE config 4, the configuration the metric's "1/2/4/8 B200" clause
is quoted on: one decode batch of 512 tokens over 1024 resident rank-32 adapters (ids
Zipf(1.0)) at 32B-class shapes, hidden 5120 and intermediate 27648.  gate/up is
column-parallel (A replicated, B output rows split over the ranks, no communication);
down is row-parallel (A input columns split, one sum of the FP32 [512 x 32] z rows over
the ranks between shrink and expand).  At N=1 this is the unsharded problem.  Every rank
routes the same seeded batch and holds its shard of one seeded global weight set.

At N=1 the line also carries ``sub``: configs 1 (Llama-3-8B decode, 256 tokens, 128
rank-16 adapters), 2 (retained-rank compact B, ranks U{4..64}) and 3 (8192-token prefill
in geometric segments, rank 64), the row-operator pair on config 1, the padded SGLang BGMV
pair (lora_shrink / lora_expand) and the vLLM BGMV pair (vllm_gemv.shrink / expand) on config 1,
and the reference's own CUDA row kernels on config 1 (built for sm_100a into oracle/_ref: the
bar on the same box),
and on config 3 the base projection with the LoRA delta in one GEMM (lora_base_gemm) next to
cuBLAS's base GEMM followed by lora_shrink_expand_prefill, each timed the same way with its
own roofline, e2e, CPU baseline and output check.  The sub-records are measured in a random
order drawn from ``--seed`` (``sub_order``) and reported in a fixed one; each record carries
the L2-flushed time and ``warm_ms_per_step``, the median of five unflushed trials.

``value``   tokens/s of the step replayed as a CUDA graph with inputs resident in HBM
            (L2 flushed by a 256 MiB write before every timed step, outside the step's
            CUDA events), total time of exactly K steps, max over ranks.
``e2e``     the same step through the public Python API with pinned host buffers: H2D of
            the step's activations and routing, D2H of every output, per step; copies on
            their own streams with double-buffered inputs and outputs, so one step's copies
            overlap its neighbours' kernels.
``roofline`` the dominant call's algorithmic bytes / its mean CUDA-event time against the
            measured HBM copy bandwidth (MEASURED_PEAKS.json), with its ncu DRAM traffic.
``cpu_baseline`` the FP32 einsum over per-adapter gathers (the oracle port of the
            reference's torch path) on all host cores, bounded sample (rank 0, N=1).
``check``   one eager step from a zero output against the FP32 oracle (BASELINE's gate:
            max|out - ref| beyond the BF16 rounding <= 1e-2 RMS); at N>1 every rank
            checks its own output shard and the result is the AND over ranks.

Weights of the slots a batch touches are generated on the host from per-slot seeds, so
``--impl reference`` (the oracle port on the host cores, rank 0 only) computes on exactly
the same values without loading this repository's package or library; untouched slots
are filled on the device (never read by any kernel).
"""

from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "multi-LoRA shrink+expand tokens/s"
# Paths that round z (and the scaled delta) to BF16, held to the reference's gate for its row
# operators (relative L2 < 0.005) instead of BASELINE's FP32 gate.
ROUNDED_Z_PATHS = ("rows", "reference_cuda", "bgmv")
L2_NOTE = "flushed before every timed step (256 MiB write, outside the step events)"

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the dominant
# call, from one ncu capture per (config, path, call); the commands are in profiles/.
TRAFFIC = {
    (1, "fused", "gate_up_proj.fused"): (19.434496 + 75.373056 + 0.404224) * 1e6,
    (2, "fused", "proj.fused"): (51.122176 + 0.006656 + 49.678592 + 0.019456) * 1e6,
    (4, "fused", "gate_up_proj.fused"): (145.565696 + 0.168192 + 820.420352 + 53.785344) * 1e6,
    (1, "bgmv", "gate_up_proj.expand"): (75.263232 + 1.180416) * 1e6,
    (1, "vllm", "gate_up_proj.expand"): (75.279104 + 1.009920) * 1e6,
}


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", type=int, choices=(1, 2, 3, 4), default=4)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--path", choices=("fused", "rows", "bgmv", "vllm", "base_gemm", "base_cublas"),
                   default="fused")
    p.add_argument("--allreduce", choices=("peer", "nccl"), default="peer",
                   help="tensor-parallel z sum: one kernel over NVLink peer memory, or NCCL")
    p.add_argument("--no-sub", action="store_true", help="skip the config 1-3 sub-records")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-check", action="store_true")
    p.add_argument("--profile", action="store_true", help="short run for ncu (no sampling/baselines)")
    return p.parse_args(argv)


# ----------------------------------------------------------------------------- configs
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


# shapes and distributions.  Projections are (name, in_dim, slice
# widths, tensor-parallel role); roles only matter for the sharded config.
CONFIGS = {
    1: dict(
        workload="config1: decode BGMV, Llama-3-8B qkv/gate_up/down, 256 tokens, 128 adapters "
        "r=16, Zipf(1.1)",
        tokens=256, slots=128, cap=16,
        projections=(("qkv_proj", 4096, (4096, 1024, 1024), None),
                     ("gate_up_proj", 4096, (14336, 14336), None),
                     ("down_proj", 14336, (4096,), None)),
    ),
    2: dict(
        workload="config2: retained-rank decode, 512 tokens, 256 adapters, ranks U{4..64}, "
        "compact B, rsLoRA alpha=16, 4096->4096",
        tokens=512, slots=256, cap=64, projections=(("proj", 4096, (4096,), None),),
    ),
    3: dict(
        workload="config3: prefill SGMV, 8192 tokens in 32 geometric segments (mean 256), "
        "64 adapters r=64, 5120->5120",
        tokens=8192, slots=64, cap=64, projections=(("proj", 5120, (5120,), None),), prefill=True,
    ),
    4: dict(
        workload="config4: tensor-parallel decode, hidden 5120, intermediate 27648, 512 tokens, "
        "1024 adapters r=32, Zipf(1.0); gate/up column-parallel, down row-parallel with a sum "
        "of the FP32 z rows over the ranks",
        tokens=512, slots=1024, cap=32, sharded=True,
        projections=(("gate_up_proj", 5120, (27648, 27648), "column"),
                     ("down_proj", 27648, (5120,), "row")),
    ),
}


def config_routing(config, rng):
    """Per-slot ranks, scales and the token -> slot routing of a config (same on every rank)."""
    c = CONFIGS[config]
    T, G = c["tokens"], c["slots"]
    if config == 1:
        ranks, scales, slots = np.full(G, 16), np.full(G, 2.0), zipf_slots(rng, T, G, 1.1)
    elif config == 4:
        ranks, scales, slots = np.full(G, 32), np.full(G, 2.0), zipf_slots(rng, T, G, 1.0)
    elif config == 2:
        ranks = rng.choice([4, 8, 16, 32, 64], size=G)
        scales = 16.0 / np.sqrt(ranks)
        slots = rng.integers(0, G, size=T).astype(np.int32)
    else:
        ranks, scales = np.full(G, 64), np.full(G, 2.0)
        lengths = geometric_segments(rng, T, 32, 256)
        owners = rng.integers(0, G, size=len(lengths))
        slots = np.repeat(owners, lengths).astype(np.int32)
    return ranks.astype(np.int32), scales.astype(np.float32), slots


def config_record(config, world):
    """The `config` object of the JSON line (identical for both --impl arms)."""
    c = CONFIGS[config]
    sharded = c.get("sharded", False)
    return {
        "workload": c["workload"],
        "tokens": c["tokens"],
        "adapters": c["slots"],
        "rank_capacity": c["cap"],
        "l2": L2_NOTE,
        "parallelism": f"tp{world}" if sharded else f"replicas{world}",
    }


def slot_seed(seed, projection, slot):
    return (seed * 1_000_003 + projection * 100_003 + slot) % (1 << 62)


# ----------------------------------------------------------------------------- host data
class HostProjection:
    """Global (unsharded) weights of the slots one batch touches, generated on the host.

    Slot g of projection i draws A_g ~ N(0, 1/K) [S*cap, K] and B_g ~ N(0, 1/r) [N, bucket]
    (zero beyond the slot's rank) from a generator seeded by (seed, i, g), so any process
    reproduces them without a GPU.
    """

    def __init__(self, index, name, k, widths, role, ranks, cap, touched, seed):
        import torch

        self.index, self.name, self.K, self.widths, self.role = index, name, k, tuple(widths), role
        self.S, self.N, self.cap = len(widths), sum(widths), cap
        self.ranks = ranks
        self.buckets = np.array([next_pow2(r) for r in ranks])
        self.a, self.b = {}, {}
        for g in touched:
            gen = torch.Generator().manual_seed(slot_seed(seed, index, int(g)))
            r, bucket = int(ranks[g]), int(self.buckets[g])
            self.a[int(g)] = (torch.randn(self.S * cap, k, generator=gen) / k**0.5).bfloat16()
            b = torch.randn(self.N, bucket, generator=gen) / r**0.5
            b[:, r:] = 0
            self.b[int(g)] = b.bfloat16()


class HostWorkload:
    """One config's batch on the host: routing, activations, touched-slot weights."""

    def __init__(self, config, seed):
        import torch

        c = CONFIGS[config]
        rng = np.random.default_rng(seed)
        self.config, self.seed = config, seed
        self.T, self.nslots, self.cap = c["tokens"], c["slots"], c["cap"]
        self.prefill, self.sharded = c.get("prefill", False), c.get("sharded", False)
        self.ranks_np, self.scales_np, self.slots_np = config_routing(config, rng)
        self.touched = np.unique(self.slots_np[self.slots_np >= 0])
        self.t_active = int((self.slots_np >= 0).sum())
        self.x = {}
        for i, (_, k, _, _) in enumerate(c["projections"]):
            if k not in self.x:
                gen = torch.Generator().manual_seed(slot_seed(seed, 1000 + i, 0))
                self.x[k] = torch.randn(self.T, k, generator=gen).bfloat16()
        self.projections = [
            HostProjection(i, n, k, w, role, self.ranks_np, self.cap, self.touched, seed)
            for i, (n, k, w, role) in enumerate(c["projections"])
        ]


def shard_spec(hp, rank, world):
    """(input columns [lo, hi), output rows of B in shard order, shard slice widths)."""
    if hp.role is None or world == 1:
        return (0, hp.K), np.arange(hp.N), hp.widths
    if hp.role == "column":
        k_range = (0, hp.K)
    else:
        share = hp.K // world
        k_range = (rank * share, (rank + 1) * share)
    rows, widths, start = [], [], 0
    for w in hp.widths:
        share = w // world
        rows.append(np.arange(start + rank * share, start + (rank + 1) * share))
        widths.append(share)
        start += w
    return k_range, np.concatenate(rows), tuple(widths)


# ----------------------------------------------------------------------------- device data
class Projection:
    """One rank's shard of a LoRA projection on the device: packed A, compact B, metadata."""

    def __init__(self, hp, host, rank, world, device, gen):
        import torch

        (k0, k1), rows, widths = shard_spec(hp, rank, world)
        self.host, self.name, self.role = hp, hp.name, hp.role
        self.k_range, self.rows, self.widths = (k0, k1), rows, widths
        self.K, self.S, self.N, self.cap = k1 - k0, len(widths), int(sum(widths)), hp.cap
        self.ranks_np, self.scales_np = host.ranks_np, host.scales_np
        G, S, N, K, cap = host.nslots, self.S, self.N, self.K, hp.cap
        rows_t = torch.from_numpy(rows)
        # A: untouched slots random on the device, touched slots from the host set.
        self.a = torch.randn(G, S * cap, K, generator=gen, device=device, dtype=torch.bfloat16)
        self.a.mul_(hp.K**-0.5)
        idx = torch.tensor(host.touched, dtype=torch.int64)
        stack = torch.stack([hp.a[int(g)][:, k0:k1] for g in host.touched])
        self.a[idx.to(device)] = stack.to(device)
        buckets = hp.buckets
        sizes = (N * buckets + 7) // 8 * 8
        offsets = np.concatenate(([0], np.cumsum(sizes)[:-1])).astype(np.int64)
        self.b = torch.randn(int(sizes.sum()), generator=gen, device=device, dtype=torch.bfloat16)
        self.b.mul_(0.25)
        for g in host.touched:
            g = int(g)
            block = hp.b[g].index_select(0, rows_t).reshape(-1)
            self.b[offsets[g] : offsets[g] + block.numel()].copy_(block)
        self.offsets_np, self.buckets_np = offsets, buckets
        self.b_offsets = torch.tensor(offsets, dtype=torch.int64, device=device)
        self.b_strides = torch.tensor(buckets, dtype=torch.int32, device=device)
        self.ranks = torch.tensor(self.ranks_np, dtype=torch.int32, device=device)
        self.scales = torch.tensor(self.scales_np, dtype=torch.float32, device=device)
        self.slice_offsets = torch.tensor(np.cumsum((0, *widths)), dtype=torch.int32, device=device)
        self.z = torch.zeros(host.T, S * cap, dtype=torch.bfloat16, device=device)
        self.y = torch.zeros(host.T, N, dtype=torch.bfloat16, device=device)
        self.workspace = None  # sized by the workload (needs the library)

    # Algorithmic bytes (the rank-r intermediate's round trip is not counted).
    def shrink_bytes(self, touched, t_active):
        return t_active * self.K * 2 + int(self.ranks_np[touched].sum()) * self.S * self.K * 2

    def expand_bytes(self, touched, t_active):
        return int(self.buckets_np[touched].sum()) * self.N * 2 + t_active * self.N * 2 * 2

    def flops(self, slots):
        r = self.ranks_np[slots[slots >= 0]]
        return int((2 * r * (self.S * self.K + self.N)).sum())


class Workload:
    """A host batch placed on one rank's device, with the buffers the step writes."""

    def __init__(self, host, device, rank=0, world=1, path="fused"):
        import torch

        from loraforge_b200.ops.fused import prefill_workspace_floats, workspace_floats
        from loraforge_b200.ops.grouping import empty_routing

        self.host, self.config, self.device = host, host.config, device
        self.rank, self.world, self.path = rank, world, path
        self.T, self.nslots = host.T, host.nslots
        self.prefill, self.sharded = host.prefill, host.sharded
        self.ranks_np, self.scales_np, self.slots_np = host.ranks_np, host.scales_np, host.slots_np
        self.touched, self.t_active = host.touched, host.t_active
        gen = torch.Generator(device=device).manual_seed(host.seed * 7 + 11)
        self.projections = [Projection(hp, host, rank, world, device, gen) for hp in host.projections]
        self.x = {}
        for p in self.projections:
            key = (p.host.K, *p.k_range)
            if key not in self.x:
                self.x[key] = host.x[p.host.K][:, p.k_range[0] : p.k_range[1]].contiguous().to(device)
        sizer = prefill_workspace_floats if self.prefill and path in ("fused", "base_cublas") else workspace_floats
        for p in self.projections:
            p.workspace = torch.zeros(sizer(self.T, p.K, p.S, p.cap), dtype=torch.float32, device=device)
        if path in ("base_gemm", "base_cublas"):
            # The base projection W [N, K] the LoRA delta is added to (seeded on the device).
            from loraforge_b200.ops.fused import base_gemm_workspace_floats

            for p in self.projections:
                p.w = torch.randn(p.N, p.K, generator=gen, device=device, dtype=torch.bfloat16)
                p.w.mul_(p.K**-0.5)
                p.gemm_ws = torch.zeros(base_gemm_workspace_floats(self.T, p.K, p.S, p.cap), dtype=torch.float32,
                                        device=device)
        if path in ("bgmv", "vllm"):
            # The padded BGMV layouts: B as [slots, N, capacity] (the compact store when every
            # slot's bucket is the capacity) and, for vLLM, per-slice views of A and B.
            for p in self.projections:
                G = self.nslots
                if not (p.buckets_np == p.cap).all() or not (self.ranks_np == p.cap).all():
                    raise ValueError(f"--path {path} needs every slot at the full rank capacity")
                p.b_pad = p.b[: G * p.N * p.cap].view(G, p.N, p.cap)
                cols = np.cumsum((0, *p.widths))
                p.a_slices = [p.a[:, s * p.cap : (s + 1) * p.cap, :] for s in range(p.S)]
                p.b_slices = [p.b_pad[:, int(cols[s]) : int(cols[s + 1]), :] for s in range(p.S)]
                p.v = torch.zeros(p.S, self.T, p.cap, dtype=torch.float32, device=device)
            if path == "vllm" and len(set(self.scales_np.tolist())) != 1:
                raise ValueError("--path vllm takes one scale for every slot")
        self.slots = torch.from_numpy(self.slots_np).to(device)
        self.routing = empty_routing(self.T, device)
        self.peer = None

    def x_of(self, p):
        return self.x[(p.host.K, *p.k_range)]

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
    ``"bgmv"``: lora_shrink + lora_expand per projection (the padded SGLang BGMV operators, B as
    [slots, N, capacity]); ``"vllm"``: vllm_gemv.shrink + expand per projection (vLLM's
    per-slice padded tensors, FP32 intermediate);
    ``"reference_cuda"``: the same pair run by the reference's own CUDA kernels, built for
    sm_100a into oracle/_ref (a comparison bar on the same box, never this repository's path);
    tensor-parallel configs: gate/up column-parallel, down as shrink, sum of the z rows
    over the ranks, expand.  ``mark(label)``, when given, records a CUDA event that starts
    the interval named `label` (ended by the next mark or "end").
    """
    from loraforge_b200.ops import lora_expand, lora_shrink, row_expand, row_shrink, vllm_gemv
    from loraforge_b200.ops.fused import (
        lora_base_gemm,
        lora_shrink_expand,
        lora_shrink_expand_prefill,
        sgmv_expand,
        sgmv_shrink,
        z_rows,
    )
    from loraforge_b200.ops.grouping import group_tokens

    mark = mark or (lambda label: None)
    prefill = w.prefill and w.path in ("fused", "base_gemm", "base_cublas")
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
        if p.role == "row" and w.world > 1:
            mark(f"{p.name}.shrink")
            sgmv_shrink(x, p.a, p.b, p.y, workspace=p.workspace, **meta, num_slices=p.S)
            mark(f"{p.name}.allreduce")
            z = z_rows(p.workspace, w.T, p.K, p.S, p.cap)
            if w.peer is not None:
                w.peer(z)
            else:
                import torch.distributed as dist

                dist.all_reduce(z)
            mark(f"{p.name}.expand")
            sgmv_expand(x, p.a, p.b, p.y, workspace=p.workspace, **meta, num_slices=p.S)
        elif w.path == "fused":
            mark(f"{p.name}.fused")
            fused_op(x, p.a, p.b, p.y, **meta, num_slices=p.S, workspace=p.workspace)
        elif w.path == "base_gemm":
            mark(f"{p.name}.gemm")
            lora_base_gemm(x, p.w, p.a, p.b, p.y, **meta, num_slices=p.S, slice_widths=p.widths,
                           workspace=p.gemm_ws)
        elif w.path == "base_cublas":
            import torch

            mark(f"{p.name}.gemm")
            torch.matmul(x, p.w.t(), out=p.y)
            mark(f"{p.name}.fused")
            lora_shrink_expand_prefill(x, p.a, p.b, p.y, **meta, num_slices=p.S, workspace=p.workspace)
        elif w.path == "reference_cuda":
            mark(f"{p.name}.shrink")
            w.ref.shrink(x, p.a, p.z, w.slots, p.ranks, p.S, p.cap)
            mark(f"{p.name}.expand")
            w.ref.expand(p.z, p.b, p.b_offsets, p.b_strides, p.y, r.segment_indptr, r.segment_slots,
                         r.token_indices, p.ranks, p.scales, p.slice_offsets, r.segment_count, p.N, p.cap,
                         2 * w.sms, 256)
        elif w.path == "bgmv":
            mark(f"{p.name}.shrink")
            z = lora_shrink(x, p.a, p.ranks, w.slots, num_slices=p.S)
            mark(f"{p.name}.expand")
            lora_expand(z, p.b_pad, p.ranks, p.scales, w.slots, p.slice_offsets, max(p.widths), base=p.y)
        elif w.path == "vllm":
            mark(f"{p.name}.shrink")
            vllm_gemv.shrink(x, p.a_slices, p.v, w.slots, scale=float(w.scales_np[0]))
            mark(f"{p.name}.expand")
            vllm_gemv.expand(p.v, p.b_slices, p.y, w.slots, offset=0, add=True)
        else:
            mark(f"{p.name}.shrink")
            row_shrink(x, p.a, p.z, w.slots, p.ranks, num_slices=p.S, max_rank=p.cap)
            mark(f"{p.name}.expand")
            row_expand(p.z, p.b, p.y, **meta)
    mark("end")


def launches_per_step(w):
    """This library's kernels per step: grouping, two per projection, the peer z sum."""
    if w.path == "reference_cuda":
        return 1  # only the grouping is this library's
    peer = 1 if (w.peer is not None and any(p.role == "row" for p in w.projections)) else 0
    return 1 + 2 * len(w.projections) + peer


# ----------------------------------------------------------------------------- checks
def oracle_delta(host, p, x_global):
    """FP32 oracle delta of this rank's output shard of projection `p` (host tensors)."""
    import torch

    from oracle.cpu_reference import lora_delta_fp32

    hp = p.host
    rows_t = torch.from_numpy(p.rows)

    def b_rows(g):
        return hp.b[int(g)].index_select(0, rows_t)

    return lora_delta_fp32(x_global.float(), hp.a, b_rows, host.slots_np, host.ranks_np,
                           host.scales_np, p.slice_offsets.cpu().numpy())


def check_outputs(w):
    """One eager step from zero outputs against the FP32 oracle.

    Fused paths (FP32 z): BASELINE's gate, max|out - ref| beyond the BF16 rounding of the
    output <= 1e-2 RMS.  The row-operator pair rounds z and the scaled delta to BF16 (the
    retained-rank contract), so it is held to the reference's own gate for that pair,
    relative L2 < 0.005.  Returns (ok, worst figures over the projections).
    """
    import torch

    from oracle.cpu_reference import fp32_gate

    for p in w.projections:
        p.y.zero_()
    run_step(w)
    torch.cuda.synchronize()
    worst = {"excess": 0.0, "raw": 0.0, "exact": 1.0, "rel_l2": 0.0}
    for p in w.projections:
        expected = oracle_delta(w.host, p, w.host.x[p.host.K])
        if w.path in ("base_gemm", "base_cublas"):  # plus the base projection, FP32 on the GPU
            prev = torch.backends.cuda.matmul.allow_tf32
            torch.backends.cuda.matmul.allow_tf32 = False
            expected = expected + (w.x_of(p).float() @ p.w.float().t()).cpu().numpy()
            torch.backends.cuda.matmul.allow_tf32 = prev
        got = p.y.float().cpu().numpy()
        gate = fp32_gate(got, expected)
        gate["rel_l2"] = float(np.linalg.norm(got - expected) / max(np.linalg.norm(expected), 1e-30))
        worst = {"excess": max(worst["excess"], gate["excess"]), "raw": max(worst["raw"], gate["raw"]),
                 "exact": min(worst["exact"], gate["exact"]), "rel_l2": max(worst["rel_l2"], gate["rel_l2"])}
    ok = worst["rel_l2"] < 0.005 if w.path in ROUNDED_Z_PATHS else worst["excess"] <= 1e-2
    return ok, worst


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


def measured_tensor_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def capture(w):
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
    return graph


def time_graph(w, steps, warmup, flush, world=1):
    """Replay the captured step: exactly `steps` timed replays, L2 flushed before each.

    Returns the per-step event times (ms), the warm (unflushed) per-step median of five
    trials, and the per-interval breakdown of eager steps (mean ms per labelled call).
    """
    import torch

    graph = capture(w)
    for _ in range(warmup):
        flush.zero_()
        graph.replay()
    barrier(world)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        starts[i].record()
        graph.replay()
        ends[i].record()
    barrier(world)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    # Warm: back-to-back replays, five trials, median per-step time.
    trials = []
    reps = max(5, min(50, steps))
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        trials.append(e0.elapsed_time(e1) / reps)
    del graph
    # Kernel breakdown: eager launches queued behind a device sleep so that host launch
    # latency never shows up between the events; L2 flushed before each step.
    per_kernel = {}
    for _ in range(min(steps, 30)):
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
    return step_ms, statistics.median(trials), {k: statistics.mean(v) for k, v in per_kernel.items()}


def time_e2e(w, steps, warmup):
    """Public API with host buffers: H2D inputs, the step, D2H outputs, every step.

    Served steps are pipelined the way an engine runs them: the inputs and outputs are double
    buffered on the device and in pinned host memory, the H2D copies run on one stream, the
    step on the current stream and the D2H copies on a third, so step i's D2H and step i+1's
    H2D overlap step i+1's kernels.  Every step still copies all of its inputs in and all of its
    outputs out; the time is from the first copy to the last byte back.
    """
    import torch

    compute = torch.cuda.current_stream()
    h2d_stream, d2h_stream = torch.cuda.Stream(), torch.cuda.Stream()
    own_x, own_slots = w.x, w.slots
    own_y = [p.y for p in w.projections]
    dev_x = [own_x, {k: torch.empty_like(v) for k, v in own_x.items()}]
    dev_slots = [own_slots, torch.empty_like(own_slots)]
    dev_y = [own_y, [torch.empty_like(y).copy_(y) for y in own_y]]
    host_x = {k: v.cpu().pin_memory() for k, v in own_x.items()}
    host_slots = own_slots.cpu().pin_memory()
    host_out = [[torch.empty(y.shape, dtype=y.dtype).pin_memory() for y in own_y] for _ in range(2)]
    h2d = sum(t.numel() * 2 for t in host_x.values()) + host_slots.numel() * 4
    d2h = sum(t.numel() * 2 for t in host_out[0])
    inputs_used = [None, None]  # step done with buffer b's inputs (next H2D into b waits)
    outputs_read = [None, None]  # D2H done with buffer b's outputs (next step into b waits)

    def one(i):
        b = i % 2
        with torch.cuda.stream(h2d_stream):
            if inputs_used[b] is not None:
                h2d_stream.wait_event(inputs_used[b])
            for k, t in host_x.items():
                dev_x[b][k].copy_(t, non_blocking=True)
            dev_slots[b].copy_(host_slots, non_blocking=True)
            landed = torch.cuda.Event()
            landed.record(h2d_stream)
        compute.wait_event(landed)
        if outputs_read[b] is not None:
            compute.wait_event(outputs_read[b])
        w.x, w.slots = dev_x[b], dev_slots[b]
        for p, y in zip(w.projections, dev_y[b]):
            p.y = y
        run_step(w)
        done = torch.cuda.Event()
        done.record(compute)
        inputs_used[b] = done
        with torch.cuda.stream(d2h_stream):
            d2h_stream.wait_event(done)
            for y, h in zip(dev_y[b], host_out[b]):
                h.copy_(y, non_blocking=True)
            read = torch.cuda.Event()
            read.record(d2h_stream)
        outputs_read[b] = read

    try:
        for i in range(warmup):
            one(i)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(h2d_stream)
        for i in range(steps):
            one(i)
        compute.wait_stream(d2h_stream)
        end.record(compute)
        torch.cuda.synchronize()
    finally:
        w.x, w.slots = own_x, own_slots
        for p, y in zip(w.projections, own_y):
            p.y = y
    return start.elapsed_time(end) / steps, h2d, d2h


def cpu_baseline(host, budget_s=12.0, max_steps=50):
    """FP32 einsum over per-adapter gathers on the host (oracle port), bounded sample."""
    import torch

    from oracle.cpu_reference import lora_delta_fp32

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    xs = {k: v.float() for k, v in host.x.items()}

    def step():
        for hp in host.projections:
            lora_delta_fp32(xs[hp.K], hp.a, lambda g, hp=hp: hp.b[int(g)], host.slots_np,
                            host.ranks_np, host.scales_np, np.cumsum((0, *hp.widths)))

    t0 = time.perf_counter()
    step()  # warm-up (also sizes the sample)
    first = time.perf_counter() - t0
    times = []
    begin = time.perf_counter()
    while time.perf_counter() - begin < budget_s and len(times) < max_steps:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if first > budget_s:
            break
    per_step = statistics.median(times)
    return {
        "value": host.T / per_step,
        "unit": "tokens/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{len(times)} full steps ({len(host.projections)} projections x {host.T} tokens, "
        "unsharded), median",
    }


# ----------------------------------------------------------------------------- distributed
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


def reduce_over_ranks(value, world, op="max"):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.MIN)
    return float(t.item())


def barrier(world):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


# ----------------------------------------------------------------------------- one record
def measure(config, args, world, rank, local, path="fused", sub=False):
    """Time one config on this rank; returns the JSON record (rank 0's values are final)."""
    import torch

    device = torch.device("cuda", local)
    host = HostWorkload(config, args.seed)
    w = Workload(host, device, rank, world, path)
    if path == "reference_cuda":
        from oracle.build_ref import load

        w.ref = load("lf_ref_rows")
        if w.ref is None:
            return {"unavailable": "oracle/_ref not built (python oracle/build_ref.py)"}
        w.sms = torch.cuda.get_device_properties(device).multi_processor_count
    if w.sharded and world > 1 and args.allreduce == "peer":
        from loraforge_b200.ops.fused import z_rows
        from loraforge_b200.ops.sharded import PeerAllReduce

        down = next(p for p in w.projections if p.role == "row")
        w.peer = PeerAllReduce(z_rows(down.workspace, w.T, down.K, down.S, down.cap).numel(), device=device)
    record = {}
    if not args.no_check and not args.profile:
        ok, gate = check_outputs(w)
        ok = reduce_over_ranks(1.0 if ok else 0.0, world, op="min") == 1.0
        record["check"] = {"result": "pass" if ok else "fail",
                           "gate": ("relative L2 < 0.005 vs FP32 oracle" if path in ROUNDED_Z_PATHS else
                                    "max|out-ref| beyond BF16 rounding <= 1e-2 RMS vs FP32 oracle"),
                           "excess": reduce_over_ranks(gate["excess"], world),
                           "raw": reduce_over_ranks(gate["raw"], world),
                           "exact": reduce_over_ranks(gate["exact"], world, op="min"),
                           "rel_l2": reduce_over_ranks(gate["rel_l2"], world)}
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    steps, warmup = args.steps, max(3, args.warmup)
    barrier(world)
    with ClockSampler(local) as clocks:
        step_ms, warm_ms, per_kernel = time_graph(w, steps, warmup, flush, world)
    total_ms = reduce_over_ranks(sum(step_ms), world)
    ms_per_step = total_ms / steps
    # Replicas: every rank processes its own batch; tensor-parallel: the ranks share one.
    tokens_per_step = (1 if w.sharded else world) * w.T
    value = tokens_per_step * steps / (total_ms / 1e3)
    peak, peak_kind = measured_peaks()
    kernels = {k: v for k, v in per_kernel.items() if k.split(".")[1] in ("shrink", "expand", "fused", "gemm")}
    dominant = max(kernels, key=kernels.get)
    name, kind = dominant.split(".")
    p = next(p for p in w.projections if p.name == name)
    if kind == "gemm":  # the base projection GEMM: tensor-bound, FLOPs of base plus LoRA
        alg = 2 * w.T * p.K * p.N + (p.flops(w.slots_np) if path == "base_gemm" else 0)
        achieved = alg / (per_kernel[dominant] * 1e-3) / 1e12
        peak, peak_kind = measured_tensor_peak()
    else:
        alg = {
            "shrink": p.shrink_bytes(w.touched, w.t_active),
            "expand": p.expand_bytes(w.touched, w.t_active),
            "fused": p.shrink_bytes(w.touched, w.t_active) + p.expand_bytes(w.touched, w.t_active),
        }[kind]
        achieved = alg / (per_kernel[dominant] * 1e-3) / 1e9
    record.update({
        "value": value,
        "unit": "tokens/s",
        "ms_per_step": ms_per_step,
        "warm_ms_per_step": reduce_over_ranks(warm_ms, world),
        "config": config_record(config, world),
        "path": path,
        "hbm_gbs_step": w.bytes_per_step() / (ms_per_step * 1e-3) / 1e9,
        "bytes_per_step": w.bytes_per_step(),
        "flops_per_step": w.flops_per_step(),
        "kernel_ms": per_kernel,
        "roofline": {
            "bound": "tensor" if kind == "gemm" else "hbm",
            "kernel": dominant,
            "achieved": achieved,
            "peak": peak,
            "unit": "TFLOP/s" if kind == "gemm" else "GB/s",
            "frac": achieved / peak,
            "peak_source": (
                f"measured (MEASURED_PEAKS.json {'bf16_tflops' if kind == 'gemm' else 'hbm_gbs'})"
                if peak_kind == "measured"
                else "fallback (no MEASURED_PEAKS.json: earlier measurement on this pool, "
                + ("1.59 PFLOP/s cuBLAS BF16 burst)" if kind == "gemm" else "6.65 TB/s copy)")
            ),
            "alg_flops" if kind == "gemm" else "alg_bytes": alg,
            "traffic": TRAFFIC.get((config, path, dominant)),
        },
        "gpu_launches": launches_per_step(w) * steps,
        "clocks": clocks.record(),
    })
    if w.sharded and world > 1:
        record["config"]["z_sum"] = args.allreduce
    if not args.no_e2e and not args.profile:
        e2e_ms, h2d, d2h = time_e2e(w, max(10, steps // 10), 3)
        e2e_ms = reduce_over_ranks(e2e_ms, world)
        record["e2e"] = {
            "value": tokens_per_step / (e2e_ms * 1e-3),
            "unit": "tokens/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
        }
    if "down_proj.allreduce" in per_kernel:  # the z sum, timed on its own
        record["allreduce_us"] = reduce_over_ranks(per_kernel["down_proj.allreduce"], world) * 1e3
    if (rank == 0 and world == 1 and not args.no_cpu_baseline and not args.profile
            and path not in ("reference_cuda", "bgmv", "vllm", "base_gemm", "base_cublas")):
        record["cpu_baseline"] = cpu_baseline(host, budget_s=8.0 if sub else 12.0)
    if path == "reference_cuda":
        record["impl"] = "reference CUDA kernels (src/loraforge/ops/csrc/lora_rows.cu, sm_100a, oracle/_ref)"
    if w.peer is not None:
        w.peer.close()
    del w, flush
    torch.cuda.empty_cache()
    return record


# ----------------------------------------------------------------------------- sub-records
SUB_RECORDS = ((1, "fused"), (2, "fused"), (3, "fused"), (1, "rows"), (1, "reference_cuda"),
               (1, "bgmv"), (1, "vllm"), (3, "base_gemm"), (3, "base_cublas"))


def sub_record_name(config, path):
    return f"config{config}" + ("" if path == "fused" else f"_{path}")


def sub_record_order(seed):
    """Indices of SUB_RECORDS in measurement order: a random order drawn from ``seed``, so that
    no variant always runs right after the same neighbour (warm clocks, L2 contents, allocator
    state); the line reports them in the fixed order."""
    order = list(range(len(SUB_RECORDS)))
    random.Random(seed).shuffle(order)
    return order


# ----------------------------------------------------------------------------- main
def main(argv=None):
    args = parse_args(argv)
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        return main_reference(args, world_env)
    import torch

    world, rank, local = init_distributed()
    torch.cuda.set_device(local)
    head = measure(args.config, args, world, rank, local, args.path)
    result = {
        "metric": METRIC,
        "value": head.pop("value"),
        "unit": head.pop("unit"),
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(3, args.warmup),
        "ms_per_step": head.pop("ms_per_step"),
        "higher_is_better": True,
        "scaling": "strong" if CONFIGS[args.config].get("sharded") else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": f"synthetic (seeded; BASELINE config {args.config} shapes and distributions)",
        "config": head.pop("config"),
    }
    result.update(head)
    if world == 1 and args.config == 4 and not args.no_sub and not args.profile:
        variants = SUB_RECORDS
        names = [sub_record_name(c, path) for c, path in variants]
        order = sub_record_order(args.seed)
        measured = {}
        for i in order:
            config, path = variants[i]
            measured[names[i]] = measure(config, args, world, rank, local, path, sub=True)
        result["sub"] = {name: measured[name] for name in names}
        result["sub_order"] = [names[i] for i in order]
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main_reference(args, world):
    """CPU oracle port of the reference path on the host cores (rank 0 only).

    Builds the same seeded batch on the host and never imports this repository's package
    or loads its library.
    """
    if int(os.environ.get("RANK", "0")) != 0:
        return
    host = HostWorkload(args.config, args.seed)
    budget = max(10.0, min(120.0, 2.0 * (args.steps + args.warmup)))
    base = cpu_baseline(host, budget_s=budget)
    print(
        json.dumps(
            {
                "impl": "reference",
                "metric": METRIC,
                "value": base["value"],
                "unit": "tokens/s",
                "n_gpus": world,
                "steps": args.steps,
                "warmup": max(3, args.warmup),
                "ms_per_step": 1e3 * host.T / base["value"],
                "higher_is_better": True,
                "scaling": "strong" if CONFIGS[args.config].get("sharded") else "weak",
                "vs_baseline": None,
                "dtype": "f32",
                "data": f"synthetic (seeded; BASELINE config {args.config} shapes and distributions)",
                "config": config_record(args.config, world),
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "tokens/s",
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            }
        ),
        flush=True,
    )


if __name__ == "__main__":
    main()
