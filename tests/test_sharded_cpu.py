"""Tensor-parallel LoRA host logic on CPU: the weight-sharding helpers and the
row-/column-parallel decomposition over two gloo ranks, with the oracle's FP32 einsum
standing in for the kernels."""

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import cpu_reference as ref  # noqa: E402

from loraforge_b200.ops.sharded import shard_a_columns, shard_b_columns, shard_bounds  # noqa: E402


def problem(seed=0, tokens=48, slots=6, k=64, widths=(32, 32), rank=8):
    g = torch.Generator().manual_seed(seed)
    S, N = len(widths), sum(widths)
    ranks = [rank] * slots
    x = torch.randn(tokens, k, generator=g)
    a = torch.randn(slots, S * rank, k, generator=g) / k**0.5
    pieces, offsets, cursor = [], [], 0
    for _ in range(slots):
        offsets.append(cursor)
        block = torch.randn(N * rank, generator=g) / rank**0.5
        pieces.append(block)
        cursor += block.numel()
    b = torch.cat(pieces)
    ids = torch.randint(-1, slots, (tokens,), generator=g).numpy()
    scales = (torch.rand(slots, generator=g) + 0.5).numpy()
    return dict(x=x, a=a, b=b, offsets=torch.tensor(offsets), strides=torch.tensor([rank] * slots),
                ranks=np.array(ranks), ids=ids, scales=scales, widths=widths)


def delta(p, x, a, b, offsets, widths):
    n = sum(widths)
    strides = p["strides"].tolist()

    def rows(g):
        off = int(offsets[g])
        return b[off : off + n * strides[g]].view(n, strides[g])

    return ref.lora_delta_fp32(x.numpy(), a, rows, p["ids"], p["ranks"], p["scales"], np.cumsum((0, *widths)))


def test_shard_bounds_and_divisibility():
    assert shard_bounds(12, 2, 4) == (6, 9)
    with pytest.raises(ValueError, match="divisible"):
        shard_bounds(10, 0, 4)
    with pytest.raises(ValueError, match="rank"):
        shard_bounds(8, 4, 4)


def test_column_shards_concatenate_to_the_full_delta():
    p = problem(seed=1)
    full = delta(p, p["x"], p["a"], p["b"], p["offsets"], p["widths"])
    world, (w0, w1) = 2, p["widths"]
    parts = []
    for r in range(world):
        b, offs, widths = shard_b_columns(p["b"], p["offsets"], p["strides"], p["widths"], r, world)
        assert all(int(o) % 8 == 0 for o in offs)
        parts.append(delta(p, p["x"], p["a"], b, offs, widths))
    # Rank r's columns of slice s sit at rank r's shard of that slice.
    got = np.concatenate([parts[0][:, : w0 // 2], parts[1][:, : w0 // 2],
                          parts[0][:, w0 // 2 :], parts[1][:, w0 // 2 :]], axis=1)
    np.testing.assert_allclose(got, full, rtol=1e-5, atol=1e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _row_parallel_worker(rank, world, port, out):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        p = problem(seed=2, widths=(32,))
        x = p["x"][:, slice(*shard_bounds(p["x"].shape[1], rank, world))]
        a = shard_a_columns(p["a"], rank, world)
        b, offs, widths = shard_b_columns(p["b"], p["offsets"], p["strides"], p["widths"], rank, world)
        # Partial z of this rank's input columns, summed over the group, then this
        # rank's output columns (the decomposition row_parallel performs on device).
        T, r = x.shape[0], int(p["ranks"][0])
        z = torch.zeros(T, r)
        for t in range(T):
            gid = int(p["ids"][t])
            if gid >= 0:
                z[t] = a[gid, :r] @ x[t]
        dist.all_reduce(z)
        y = torch.zeros(T, widths[0])
        for t in range(T):
            gid = int(p["ids"][t])
            if gid >= 0:
                rows = b[int(offs[gid]) : int(offs[gid]) + widths[0] * r].view(widths[0], r)
                y[t] = float(p["scales"][gid]) * (rows @ z[t])
        gathered = [torch.zeros_like(y) for _ in range(world)]
        dist.all_gather(gathered, y)
        if rank == 0:
            torch.save(torch.cat(gathered, dim=1), out)
    finally:
        dist.destroy_process_group()


def test_row_parallel_over_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    out = str(tmp_path / "y.pt")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.spawn(_row_parallel_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    p = problem(seed=2, widths=(32,))
    full = delta(p, p["x"], p["a"], p["b"], p["offsets"], p["widths"])
    np.testing.assert_allclose(torch.load(out).numpy(), full, rtol=1e-4, atol=1e-4)
