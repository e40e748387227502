"""Row-parallel z sums over NVLink peer memory (lf_peer_sum through PeerAllReduce) on two
GPUs, one process each: the same bits as NCCL's all-reduce (two ranks: one addition), sizes
on the vector and scalar paths, repeated calls, capture in a CUDA graph with replays that
see new values, the status word, and the full row-parallel operator against NCCL."""

import os
import socket
from datetime import timedelta

import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(
        not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="two GPUs required"
    ),
]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import json

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    results = {}
    try:
        from loraforge_b200.ops.sharded import PeerAllReduce

        peer = PeerAllReduce(4104)
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        for n in (4096, 1000, 7, 4096):
            z = torch.randn(n, generator=g, device="cuda")
            want = z.clone()
            dist.all_reduce(want)
            got = z.clone()
            peer(got)
            torch.cuda.synchronize()
            results[f"eager_{n}_{len(results)}"] = bool(torch.equal(got, want))
        # Captured once, replayed with new inputs: the epoch advances on the device.
        z = torch.zeros(4096, device="cuda")
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            peer(z)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            peer(z)
        for it in range(3):
            z.fill_(float(rank + 1 + it))
            graph.replay()
            torch.cuda.synchronize()
            results[f"graph_{it}"] = bool((z == float(sum(r + 1 + it for r in range(world)))).all())
        del graph
        results["status"] = peer.status() == 0
        results.update(_row_parallel_case(rank, world, peer))
        peer.close()
    finally:
        dist.destroy_process_group()
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(results, f)


def _row_parallel_case(rank, world, peer):
    import numpy as np
    import torch.distributed as dist

    from loraforge_b200.ops.fused import workspace_floats, z_rows
    from loraforge_b200.ops.grouping import group_tokens
    from loraforge_b200.ops.sharded import row_parallel, shard_a_columns, shard_b_columns, shard_bounds

    # The same problem on both ranks (seeded), each rank holding its shards.
    g = torch.Generator().manual_seed(7)
    tokens, slots, k, n, r = 64, 8, 2048, 1024, 32
    x = torch.randn(tokens, k, generator=g).bfloat16().cuda()
    a = (torch.randn(slots, r, k, generator=g) / k**0.5).bfloat16().cuda()
    b = (torch.randn(slots * n * r, generator=g) / r**0.5).bfloat16().cuda()
    ids = torch.from_numpy(np.random.default_rng(3).integers(-1, slots, tokens).astype(np.int32)).cuda()
    meta = dict(b_offsets=torch.arange(slots, dtype=torch.int64).cuda() * (n * r),
                b_strides=torch.full((slots,), r, dtype=torch.int32).cuda(),
                ranks=torch.full((slots,), r, dtype=torch.int32).cuda(),
                scales=torch.rand(slots, generator=g).cuda() + 0.5,
                slice_offsets=torch.tensor([0, n // world], dtype=torch.int32).cuda())
    routing = group_tokens(ids, slots, chunk=16)
    meta.update(segment_indptr=routing.segment_indptr, segment_slots=routing.segment_slots,
                token_indices=routing.token_indices, segment_count=routing.segment_count)
    xs = x[:, slice(*shard_bounds(k, rank, world))].contiguous()
    As = shard_a_columns(a, rank, world)
    bs, offs, _ = shard_b_columns(b, meta["b_offsets"], meta["b_strides"], (n,), rank, world)
    meta["b_offsets"] = offs
    base = torch.zeros(tokens, n // world, dtype=torch.bfloat16, device="cuda")
    outs = []
    for use_peer in (True, False):
        ws = torch.zeros(workspace_floats(tokens, xs.shape[1], 1, r), dtype=torch.float32, device="cuda")
        assert z_rows(ws, tokens, xs.shape[1], 1, r).numel() <= peer.capacity
        y = base.clone()
        row_parallel(xs, As, bs, y, workspace=ws, peer=peer if use_peer else None, **meta, num_slices=1)
        torch.cuda.synchronize()
        outs.append(y)
    dist.barrier()
    return {"row_parallel": bool(torch.equal(outs[0], outs[1]))}


def test_peer_sum_matches_nccl_on_two_gpus(tmp_path):
    import json

    import torch.multiprocessing as mp

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for rank in range(world):
        results = json.loads((tmp_path / f"rank{rank}.json").read_text())
        assert results and all(results.values()), (rank, results)
