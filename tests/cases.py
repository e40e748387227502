"""Seeded operator inputs for GPU parity tests (built on the target device).

``row_case`` follows the structure of the reference fixture
(tests/test_row_operators_gpu.py:40-96 of lishenghui/loraforge): mixed ranks in a
capacity-128 pool, segments of 1..16 tokens in a random permutation, one empty
segment, one base segment, scales with zero and negatives, and an output that is
a column view inside wider storage.  ``golden_row_case`` loads the committed
golden version of the same recipe.
"""

from __future__ import annotations

import numpy as np

from golden_io import bf16_bits, load, to_torch

RANKS = [1, 2, 3, 7, 16, 17, 33, 64, 0]
SIZES = [1, 2, 3, 4, 8, 16, 15, 16, 3, 2]
SCALES = [1, -0.7, 0.5, 1.25, 2, 0, 0.3, -1, 1]


def _metadata(torch, device, permutation, widths, offsets, buckets, m):
    starts, slots = [0], []
    routes = [-1] * m
    for slot, size in enumerate(SIZES):
        actual = slot if slot < len(RANKS) else -1
        slots.append(actual)
        for t in permutation[starts[-1] : starts[-1] + size]:
            routes[t] = actual
        starts.append(starts[-1] + size)
    slots += [0, -1]
    starts += [m, m]
    bounds = [0]
    for w in widths:
        bounds.append(bounds[-1] + w)

    def tensor(values, dtype=torch.int32):
        return torch.tensor(values, dtype=dtype, device=device)

    meta = dict(
        b_offsets=tensor(offsets, torch.int64),
        b_strides=tensor(buckets),
        ranks=tensor(RANKS),
        scales=tensor(SCALES, torch.float32),
        segment_indptr=tensor(starts),
        segment_slots=tensor(slots),
        token_indices=tensor(permutation),
        slice_offsets=tensor(bounds),
        segment_count=tensor([len(slots) - 1]),
    )
    return tensor(routes), meta


def row_case(slices=1, width=520, columns=None, device="cuda:0", seed=31):
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    m, capacity = sum(SIZES), 128
    widths = [19, 13, 11][:slices] if columns is None else [columns] * slices
    n = sum(widths)
    x = (torch.randn(m, width + 8, generator=g) * 0.1).bfloat16().to(device)[:, :width]
    a = (torch.randn(len(RANKS), slices * capacity, width, generator=g) * 0.1).bfloat16().to(device)
    z = torch.full((m, slices * capacity), 3.0, dtype=torch.bfloat16, device=device)
    storage = (torch.randn(m, n + 6, generator=g) * 0.1).bfloat16().to(device)
    output = storage[:, 3 : 3 + n]
    permutation = torch.randperm(m, generator=g).tolist()
    pieces, offsets, buckets, cursor = [], [], [], 0
    for rank in RANKS:
        padding = (-cursor) % 8
        pieces.append(torch.zeros(padding, dtype=torch.bfloat16))
        cursor += padding
        bucket = 1 << (max(1, rank) - 1).bit_length()
        b = (torch.randn(n, bucket, generator=g) * 0.1).bfloat16()
        b[:, rank:] = 0
        offsets.append(cursor)
        buckets.append(bucket)
        pieces.append(b.flatten())
        cursor += b.numel()
    routes, meta = _metadata(torch, device, permutation, widths, offsets, buckets, m)
    return x, a, z, torch.cat(pieces).to(device), storage, output, routes, meta


def golden_row_case(slices, device="cuda:0"):
    """The committed reference-fixture case: tensors plus the reference outputs."""
    import torch

    d = load(f"row_case_s{slices}.npz")
    m, width = d["x"].shape
    xs = torch.zeros(m, width + 8, dtype=torch.bfloat16, device=device)
    xs[:, :width] = to_torch(d["x"], device=device)
    x = xs[:, :width]
    a = to_torch(d["a"], device=device)
    z = to_torch(d["z"], device=device)
    b = to_torch(d["b"], device=device)
    storage = to_torch(d["storage"], device=device)
    lo, hi = (int(v) for v in d["output_columns"])
    output = storage[:, lo:hi]
    routes = to_torch(d["routes"], device=device)
    meta = {
        k: to_torch(d[k], device=device)
        for k in (
            "b_offsets", "b_strides", "ranks", "scales", "segment_indptr", "segment_slots",
            "token_indices", "slice_offsets", "segment_count",
        )
    }
    return (x, a, z, b, storage, output, routes, meta), d


def np_meta(meta) -> dict:
    """Device metadata as numpy (for the oracle)."""
    out = {k: v.cpu().numpy() for k, v in meta.items()}
    out["segment_count"] = int(out["segment_count"][0])
    return out


def oracle_expand(z, b, y, meta):
    """Bit-exact oracle RowExpand of device tensors; returns BF16 bits."""
    from oracle import cpu_reference as ref

    mm = np_meta(meta)
    return ref.row_expand(
        bf16_bits(z), bf16_bits(b), bf16_bits(y), mm["b_offsets"], mm["b_strides"], mm["ranks"],
        mm["scales"], mm["segment_indptr"], mm["segment_slots"], mm["token_indices"],
        mm["slice_offsets"], mm["segment_count"],
    )


def oracle_shrink(x, a, z, routes, ranks, slices, max_rank=64):
    from oracle import cpu_reference as ref

    return ref.row_shrink(
        ref.bf16_value(bf16_bits(x)), ref.bf16_value(bf16_bits(a)), bf16_bits(z),
        routes.cpu().numpy(), ranks.cpu().numpy(), slices, max_rank,
    )


def values(bits) -> np.ndarray:
    from oracle import cpu_reference as ref

    return ref.bf16_value(bits)
