"""Fleet-form direct_shrink / row_expand (positional API, up to 4 slices, row tiles).

Mirrors the kernel-level parts of tests/test_rowexpand_gpu.py in lishenghui/loraforge:
four unequal slices (:225-275) and row_tile x threads bitwise equality to tile 16
(:278-379), plus the C++ argument checks (RuntimeError, "row_tile must").
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from cases import oracle_expand, oracle_shrink, values  # noqa: E402
from golden_io import bf16_bits, rel_l2  # noqa: E402
from oracle import cpu_reference as ref  # noqa: E402

from loraforge_b200.ops.grouping import group_tokens  # noqa: E402
from loraforge_b200.ops.rowexpand import direct_shrink, row_expand, rowexpand_extension  # noqa: E402


def fleet_case(widths=(1024, 256, 512, 128), capacity=64, tokens=45, slots=6, seed=11):
    g = torch.Generator().manual_seed(seed)
    S, K, N = len(widths), 1024, sum(widths)
    ranks = [16, 64, 3, 0, 32, 7][:slots]
    x = (torch.randn(tokens, K, generator=g) * 0.1).bfloat16().cuda()
    a = (torch.randn(slots, S * capacity, K, generator=g) * 0.1).bfloat16().cuda()
    pieces, offsets, buckets, cursor = [], [], [], 0
    for r in ranks:
        cursor_pad = (-cursor) % 8
        pieces.append(torch.zeros(cursor_pad, dtype=torch.bfloat16))
        cursor += cursor_pad
        bucket = 1 << (max(1, r) - 1).bit_length()
        b = (torch.randn(N, bucket, generator=g) * 0.1).bfloat16()
        b[:, r:] = 0
        offsets.append(cursor)
        buckets.append(bucket)
        pieces.append(b.flatten())
        cursor += b.numel()
    store = torch.cat(pieces).cuda()
    routes = torch.randint(-1, slots, (tokens,), generator=g, dtype=torch.int32).cuda()
    meta = dict(
        offsets=torch.tensor(offsets, dtype=torch.int64, device="cuda"),
        buckets=torch.tensor(buckets, dtype=torch.int32, device="cuda"),
        ranks=torch.tensor(ranks, dtype=torch.int32, device="cuda"),
        scales=(torch.rand(slots, generator=g) * 2 - 1).cuda(),
        slice_offsets=torch.tensor(np.cumsum([0, *widths]), dtype=torch.int32, device="cuda"),
    )
    base = (torch.randn(tokens, N, generator=g) * 0.1).bfloat16().cuda()
    return x, a, store, routes, meta, base, S, capacity


def run_fleet(x, a, store, routes, meta, base, S, capacity, *, row_tile=16, threads=256, blocks=880):
    z = torch.zeros(x.shape[0], a.shape[1], dtype=torch.bfloat16, device="cuda")
    direct_shrink(x, a, z, routes, meta["ranks"], S, 64)
    routing = group_tokens(routes, meta["ranks"].numel(), chunk=16)
    out = base.clone()
    row_expand(
        z, store, meta["offsets"], meta["buckets"], out, routing.segment_indptr,
        routing.segment_slots, routing.token_indices, meta["ranks"], meta["scales"],
        meta["slice_offsets"], routing.segment_count, capacity,
        blocks=blocks, threads=threads, row_tile=row_tile,
    )
    return z, out, routing


def test_four_unequal_slices_against_oracle():
    rowexpand_extension()
    x, a, store, routes, meta, base, S, cap = fleet_case()
    z, out, routing = run_fleet(x, a, store, routes, meta, base, S, cap)
    torch.cuda.synchronize()
    expected_z = oracle_shrink(x, a, torch.zeros_like(z), routes, meta["ranks"], S)
    ranks = meta["ranks"].cpu().numpy()
    r = np.where(routes.cpu().numpy() >= 0, ranks[np.clip(routes.cpu().numpy(), 0, None)], 0)
    live = np.arange(z.shape[1])[None, :] < (S * r)[:, None]
    assert rel_l2(values(bf16_bits(z)[live]), values(expected_z[live])) < 0.005
    meta_np = {
        "b_offsets": meta["offsets"], "b_strides": meta["buckets"], "ranks": meta["ranks"],
        "scales": meta["scales"], "segment_indptr": routing.segment_indptr,
        "segment_slots": routing.segment_slots, "token_indices": routing.token_indices,
        "slice_offsets": meta["slice_offsets"], "segment_count": routing.segment_count,
    }
    count = int(routing.segment_count.item())
    meta_np["segment_slots"] = routing.segment_slots[:count]
    meta_np["segment_indptr"] = routing.segment_indptr[: count + 1]
    np.testing.assert_array_equal(bf16_bits(out), oracle_expand(z, store, base, meta_np))


@pytest.mark.parametrize("row_tile", [2, 4, 8])
@pytest.mark.parametrize("threads", [128, 256])
def test_row_tiles_are_bitwise_equal_to_whole_segments(row_tile, threads):
    case = fleet_case(widths=(512, 128, 128), seed=5)
    _, whole, _ = run_fleet(*case)
    _, tiled, _ = run_fleet(*case, row_tile=row_tile, threads=threads, blocks=37)
    torch.testing.assert_close(tiled, whole, rtol=0, atol=0)


def test_argument_checks_raise_runtime_error():
    x, a, store, routes, meta, base, S, cap = fleet_case()
    z = torch.zeros(x.shape[0], a.shape[1], dtype=torch.bfloat16, device="cuda")
    routing = group_tokens(routes, meta["ranks"].numel())
    args = (
        z, store, meta["offsets"], meta["buckets"], base.clone(), routing.segment_indptr,
        routing.segment_slots, routing.token_indices, meta["ranks"], meta["scales"],
        meta["slice_offsets"], routing.segment_count, cap,
    )
    with pytest.raises(RuntimeError, match="row_tile must"):
        row_expand(*args, row_tile=3)
    with pytest.raises(RuntimeError):
        row_expand(*args, threads=64)
    with pytest.raises(ValueError, match="autograd"):
        direct_shrink(x.float().requires_grad_(), a, z, routes, meta["ranks"], S, 64)
    assert ref is not None
