"""Parity at BASELINE's real configurations: every config built exactly as bench.py builds it.

Each case places bench.py's seeded batch (``HostWorkload`` -> ``Workload``) on cuda:0 and
runs one step through the public API from zero outputs:

* grouping is compared bit for bit with the CPU restatement (slot-ordered segments of 16
  tokens for decode, runs in token order cut at 128 tokens for prefill);
* every projection's output is compared with the FP32 einsum over per-adapter gathers
  (BASELINE's gate: max|out - ref| beyond the BF16 rounding <= 1e-2 RMS, and > 99% of
  outputs equal to bf16(ref)).

Config 4 is also split into two tensor-parallel shards computed on the one device: the
column-parallel gate/up per shard, the row-parallel down as shard shrinks, a sum of the two
ranks' FP32 z rows by hand, and shard expands; each shard is checked against the oracle of
its own output columns.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

import bench  # noqa: E402
from oracle import cpu_reference as ref  # noqa: E402
from test_grouping_gpu import runs_reference  # noqa: E402

from loraforge_b200.ops.fused import sgmv_expand, sgmv_shrink, z_rows  # noqa: E402

SEED = 1234  # bench.py's default seed: the timed batch itself


def _gate(p, host):
    expected = bench.oracle_delta(host, p, host.x[p.host.K])
    gate = ref.fp32_gate(p.y.float().cpu().numpy(), expected)
    assert gate["excess"] <= 1e-2, (p.name, gate)
    assert gate["exact"] > 0.99, (p.name, gate)


def _grouping_exact(w):
    r = w.routing
    count = int(r.segment_count.item())
    if w.prefill:
        want_indptr, want_slots, want_perm = runs_reference(w.slots_np, w.nslots, 128)
        want_count = len(want_slots)
    else:
        want_indptr, want_slots, want_perm, want_count = ref.group_tokens(w.slots_np, w.nslots, 16)
    assert count == want_count
    assert r.segment_indptr[: count + 1].cpu().numpy().tolist() == list(np.asarray(want_indptr).tolist())
    assert r.segment_slots[:count].cpu().numpy().tolist() == list(np.asarray(want_slots).tolist())
    assert r.token_indices[: w.T].cpu().numpy().tolist() == list(np.asarray(want_perm).tolist())


@pytest.fixture(scope="module")
def hosts():
    return {}


def _host(hosts, config):
    if config not in hosts:
        hosts[config] = bench.HostWorkload(config, SEED)
    return hosts[config]


@pytest.mark.parametrize("config", [1, 2, 3, 4])
def test_config_one_step_against_oracle(hosts, config):
    host = _host(hosts, config)
    w = bench.Workload(host, torch.device("cuda", 0))
    for p in w.projections:
        p.y.zero_()
    bench.run_step(w)
    torch.cuda.synchronize()
    _grouping_exact(w)
    for p in w.projections:
        _gate(p, host)
    # Replaying the step as a CUDA graph adds the same delta again, bit for bit.
    first = [p.y.clone() for p in w.projections]
    for p in w.projections:
        p.y.zero_()
    graph = bench.capture(w)  # three eager warm-up steps, then the capture
    for p in w.projections:
        p.y.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for p, y in zip(w.projections, first):
        assert torch.equal(p.y, y), p.name


def test_config4_two_shards_on_one_device(hosts):
    host = _host(hosts, 4)
    device = torch.device("cuda", 0)
    shards = [bench.Workload(host, device, rank, 2) for rank in range(2)]
    from loraforge_b200.ops.fused import lora_shrink_expand
    from loraforge_b200.ops.grouping import group_tokens

    metas = []
    for w in shards:
        r = group_tokens(w.slots, w.nslots, chunk=16, out=w.routing)
        metas.append(dict(segment_indptr=r.segment_indptr, segment_slots=r.segment_slots,
                          token_indices=r.token_indices, segment_count=r.segment_count))
    for w, routing in zip(shards, metas):
        for p in w.projections:
            p.y.zero_()
            meta = dict(b_offsets=p.b_offsets, b_strides=p.b_strides, ranks=p.ranks, scales=p.scales,
                        slice_offsets=p.slice_offsets, **routing)
            if p.role == "column":
                lora_shrink_expand(w.x_of(p), p.a, p.b, p.y, **meta, num_slices=p.S, workspace=p.workspace)
            else:
                sgmv_shrink(w.x_of(p), p.a, p.b, p.y, workspace=p.workspace, **meta, num_slices=p.S)
    downs = [next(p for p in w.projections if p.role == "row") for w in shards]
    zs = [z_rows(p.workspace, host.T, p.K, p.S, p.cap) for p in downs]
    total = zs[0] + zs[1]
    for z in zs:
        z.copy_(total)
    for w, routing, p in zip(shards, metas, downs):
        meta = dict(b_offsets=p.b_offsets, b_strides=p.b_strides, ranks=p.ranks, scales=p.scales,
                    slice_offsets=p.slice_offsets, **routing)
        sgmv_expand(w.x_of(p), p.a, p.b, p.y, workspace=p.workspace, **meta, num_slices=p.S)
    torch.cuda.synchronize()
    for w in shards:
        for p in w.projections:
            _gate(p, host)
