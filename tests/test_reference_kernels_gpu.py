"""This repository's row kernels against the reference's own CUDA kernels, on the B200.

The reference's ``lora_rows.cu`` and ``rowexpand.cu`` are compiled for sm_100a into
``oracle/_ref`` by ``oracle/build_ref.py`` (test infrastructure; never loaded by the
product).  On the same inputs and metadata:

* ``row_expand`` (retained-rank and fleet forms) must be bit-identical to the reference
  kernels: the arithmetic contract (FP32 multiply-add over k, BF16-rounded scaled delta,
  BF16 sum) leaves no freedom;
* ``row_shrink`` / ``direct_shrink`` sum every rank row in the reference's order (lane
  chunks, fused multiply-adds, the same shuffle tree), so their BF16 z must be bit-identical
  to the reference kernels' too, untouched entries included.

Cases: the reference fixture recipe at 1, 2 and 3 slices (mixed ranks, a base segment, an
empty segment, odd widths) and BASELINE config 1's three Llama-3-8B projections.  Only
metadata inside the reference's contract is fed to its kernels (they return early on a
contract breach, src/loraforge/ops/csrc/lora_rows.cu:139).
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.build_ref import load  # noqa: E402

REF_ROWS = load("lf_ref_rows")
REF_FLEET = load("lf_ref_rowexpand")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
    pytest.mark.skipif(REF_ROWS is None or REF_FLEET is None,
                       reason="oracle/_ref not built (python oracle/build_ref.py)"),
]

import bench  # noqa: E402
from cases import golden_row_case  # noqa: E402
from golden_io import bf16_bits  # noqa: E402

from loraforge_b200.ops import row_expand, row_shrink  # noqa: E402
from loraforge_b200.ops.grouping import group_tokens  # noqa: E402
from loraforge_b200.ops.rowexpand import direct_shrink  # noqa: E402
from loraforge_b200.ops.rowexpand import row_expand as fleet_expand  # noqa: E402


def _shrink_pair(x, a, routes, ranks, slices, max_rank=64):
    z_ref = torch.zeros(x.shape[0], a.shape[1], dtype=torch.bfloat16, device="cuda")
    z_ours = z_ref.clone()
    REF_ROWS.shrink(x, a, z_ref, routes, ranks, slices, max_rank)
    row_shrink(x, a, z_ours, routes, ranks, num_slices=slices, max_rank=max_rank)
    torch.cuda.synchronize()
    return z_ref, z_ours


def _expand_ref(z, b, y, meta, slices, blocks=296, threads=256):
    n = y.shape[1]
    REF_ROWS.expand(z, b, meta["b_offsets"], meta["b_strides"], y, meta["segment_indptr"],
                    meta["segment_slots"], meta["token_indices"], meta["ranks"], meta["scales"],
                    meta["slice_offsets"], meta["segment_count"], n, z.shape[1] // slices, blocks, threads)


@pytest.mark.parametrize("slices", [1, 2, 3])
def test_golden_cases_against_reference_kernels(slices):
    (x, a, z, b, storage, output, routes, meta), _ = golden_row_case(slices)
    z_ref, z_ours = _shrink_pair(x, a, routes, meta["ranks"], slices)
    np.testing.assert_array_equal(bf16_bits(z_ours), bf16_bits(z_ref))
    # Same z into both expands: bit-identical outputs, untouched rows and columns included.
    y_ref = storage.clone()
    y_ours = storage.clone()
    lo = output.data_ptr() - storage.data_ptr()
    cols = slice(lo // 2, lo // 2 + output.shape[1])
    _expand_ref(z_ref, b, y_ref[:, cols], meta, slices)
    row_expand(z_ref, b, y_ours[:, cols], **meta)
    torch.cuda.synchronize()
    assert torch.equal(y_ours, y_ref)


@pytest.mark.parametrize("name", ["qkv_proj", "gate_up_proj", "down_proj"])
def test_config1_projections_against_reference_kernels(name):
    host = bench.HostWorkload(1, 1234)
    w = bench.Workload(host, torch.device("cuda", 0), path="rows")
    p = next(p for p in w.projections if p.name == name)
    r = group_tokens(w.slots, w.nslots, chunk=16)
    meta = dict(b_offsets=p.b_offsets, b_strides=p.b_strides, ranks=p.ranks, scales=p.scales,
                slice_offsets=p.slice_offsets, segment_indptr=r.segment_indptr,
                segment_slots=r.segment_slots, token_indices=r.token_indices, segment_count=r.segment_count)
    z_ref, z_ours = _shrink_pair(w.x_of(p), p.a, w.slots, p.ranks, p.S, p.cap)
    np.testing.assert_array_equal(bf16_bits(z_ours), bf16_bits(z_ref))
    y0 = (torch.randn(p.y.shape, generator=torch.Generator(device="cuda").manual_seed(7), device="cuda")).bfloat16()
    y_ref, y_ours = y0.clone(), y0.clone()
    _expand_ref(z_ref, p.b, y_ref, meta, p.S)
    row_expand(z_ref, p.b, y_ours, **meta)
    torch.cuda.synchronize()
    assert torch.equal(y_ours, y_ref)


@pytest.mark.parametrize("row_tile", [2, 4, 8, 16])
def test_fleet_form_against_reference_rowexpand(row_tile):
    from test_rowexpand_gpu import fleet_case

    x, a, store, routes, meta, base, S, capacity = fleet_case()
    z_ref = torch.zeros(x.shape[0], a.shape[1], dtype=torch.bfloat16, device="cuda")
    z_ours = z_ref.clone()
    REF_FLEET.shrink(x, a, z_ref, routes, meta["ranks"], S, 64)
    direct_shrink(x, a, z_ours, routes, meta["ranks"], S, 64)
    torch.cuda.synchronize()
    live = np.zeros(z_ref.shape, dtype=bool)
    rr = meta["ranks"].cpu().numpy()
    for t, g in enumerate(routes.cpu().numpy()):
        if g >= 0:
            live[t, : S * rr[g]] = True
    np.testing.assert_array_equal(bf16_bits(z_ours)[live], bf16_bits(z_ref)[live])
    routing = group_tokens(routes, meta["ranks"].numel(), chunk=16)
    n = base.shape[1]
    y_ref, y_ours = base.clone(), base.clone()
    REF_FLEET.expand(z_ref, store, meta["offsets"], meta["buckets"], y_ref, routing.segment_indptr,
                     routing.segment_slots, routing.token_indices, meta["ranks"], meta["scales"],
                     meta["slice_offsets"], routing.segment_count, n, capacity, 880, 256, row_tile)
    fleet_expand(z_ref, store, meta["offsets"], meta["buckets"], y_ours, routing.segment_indptr,
                 routing.segment_slots, routing.token_indices, meta["ranks"], meta["scales"],
                 meta["slice_offsets"], routing.segment_count, capacity, row_tile=row_tile)
    torch.cuda.synchronize()
    assert torch.equal(y_ours, y_ref)
