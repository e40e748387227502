"""Fused shrink -> expand (lf_fused_shrink_expand) on the B200 against the oracle."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from cases import golden_row_case, oracle_expand, row_case, values  # noqa: E402
from golden_io import bf16_bits, rel_l2  # noqa: E402
from oracle import cpu_reference as ref  # noqa: E402

from loraforge_b200.ops import row_expand, row_shrink  # noqa: E402
from loraforge_b200.ops.fused import lora_shrink_expand, sgmv_expand, sgmv_shrink, workspace_floats  # noqa: E402
from loraforge_b200.ops.grouping import group_tokens  # noqa: E402

ROUTING_KEYS = ("segment_indptr", "segment_slots", "token_indices", "segment_count")


def compact_store(ranks, n, gen, buckets=None):
    pieces, offsets, strides, cursor = [], [], [], 0
    for i, r in enumerate(ranks):
        bucket = buckets[i] if buckets else 1 << (max(1, r) - 1).bit_length()
        pad = (-cursor) % 8
        pieces.append(torch.zeros(pad, dtype=torch.bfloat16))
        cursor += pad
        w = (torch.randn(n, bucket, generator=gen) / max(r, 1) ** 0.5).bfloat16()
        w[:, r:] = 0
        offsets.append(cursor)
        strides.append(bucket)
        pieces.append(w.flatten())
        cursor += w.numel()
    return torch.cat(pieces), offsets, strides


def decode_case(tokens=96, slots=24, k=4096, widths=(4096, 1024, 1024), ranks=None, seed=0,
                cap=None, inactive=0.1):
    g = torch.Generator().manual_seed(seed)
    ranks = ranks or [16] * slots
    cap = cap or max(ranks)
    S, N = len(widths), sum(widths)
    x = torch.randn(tokens, k, generator=g).bfloat16()
    a = (torch.randn(slots, S * cap, k, generator=g) / k**0.5).bfloat16()
    b, offsets, strides = compact_store(ranks, N, g)
    p = 1.0 / np.arange(1, slots + 1) ** 1.1
    rng = np.random.default_rng(seed)
    ids = rng.choice(slots, size=tokens, p=p / p.sum()).astype(np.int32)
    ids[rng.random(tokens) < inactive] = -1
    scales = (torch.rand(slots, generator=g) * 2 + 0.5).float()
    base = (torch.randn(tokens, N, generator=g) * 0.5).bfloat16()
    dev = "cuda"
    meta = dict(
        b_offsets=torch.tensor(offsets, dtype=torch.int64, device=dev),
        b_strides=torch.tensor(strides, dtype=torch.int32, device=dev),
        ranks=torch.tensor(ranks, dtype=torch.int32, device=dev),
        scales=scales.to(dev),
        slice_offsets=torch.tensor(np.cumsum((0, *widths)), dtype=torch.int32, device=dev),
    )
    slots_t = torch.from_numpy(ids).to(dev)
    routing = group_tokens(slots_t, slots, chunk=16)
    meta.update(zip(ROUTING_KEYS, routing))
    return x.to(dev), a.to(dev), b.to(dev), base.to(dev), slots_t, meta, S, cap


def fp32_reference(x, a, b, base, slots_t, meta, S):
    offs = meta["b_offsets"].cpu().numpy()
    strides = meta["b_strides"].cpu().numpy()
    ranks = meta["ranks"].cpu().numpy()
    n = base.shape[1]
    bf = b.float().cpu()

    def rows(g):
        return bf[offs[g] : offs[g] + n * strides[g]].view(n, strides[g])

    delta = ref.lora_delta_fp32(
        x.float().cpu().numpy(), a.float().cpu(), rows, slots_t.cpu().numpy(), ranks,
        meta["scales"].cpu().numpy(), meta["slice_offsets"].cpu().numpy(),
    )
    return base.float().cpu().numpy() + delta


def fused(x, a, b, out, meta, S, numerics="fp32"):
    lora_shrink_expand(x, a, b, out, **meta, num_slices=S, numerics=numerics)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize(
    "widths,k", [((4096, 1024, 1024), 4096), ((14336, 14336), 4096), ((4096,), 14336)]
)
def test_llama_projections_fp32_gate(widths, k):
    x, a, b, base, slots_t, meta, S, cap = decode_case(k=k, widths=widths)
    out = fused(x, a, b, base.clone(), meta, S)
    expected = fp32_reference(x, a, b, base, slots_t, meta, S)
    gate = ref.fp32_gate(values(bf16_bits(out)), expected)
    assert gate["excess"] <= 1e-2, gate
    assert gate["exact"] > 0.99, gate
    inactive = (slots_t < 0).cpu()
    assert torch.equal(out.cpu()[inactive], base.cpu()[inactive])


def test_heterogeneous_retained_ranks():
    ranks = [4, 8, 16, 32, 64] * 8
    x, a, b, base, slots_t, meta, S, cap = decode_case(
        tokens=160, slots=len(ranks), widths=(4096,), ranks=ranks, seed=3, inactive=0.0
    )
    out = fused(x, a, b, base.clone(), meta, S)
    expected = fp32_reference(x, a, b, base, slots_t, meta, S)
    gate = ref.fp32_gate(values(bf16_bits(out)), expected)
    assert gate["excess"] <= 1e-2, gate


@pytest.mark.parametrize("slices", [1, 2, 3])
def test_reference_numerics_on_golden_cases(slices):
    (x, a, z, b, storage, output, routes, meta), gold = golden_row_case(slices)
    # The fused kernel wants an 8-byte aligned output with a row stride multiple of 4.
    n = output.shape[1]
    wide = torch.zeros(output.shape[0], (n + 3) // 4 * 4 + 4, dtype=torch.bfloat16, device="cuda")
    out = wide[:, :n]
    out.copy_(output)
    before = out.clone()
    fused(x, a, b, out, meta, slices, numerics="reference")
    assert rel_l2(values(bf16_bits(out)), values(gold["expected_y"])) < 0.005
    routes_np = gold["routes"]
    skipped = (routes_np == -1) | (routes_np == 8)
    np.testing.assert_array_equal(bf16_bits(out)[skipped], bf16_bits(before)[skipped])


@pytest.mark.parametrize("numerics", ["fp32", "reference"])
@pytest.mark.parametrize(
    "k,widths,rank",
    [(1024, (1024,), 16), (8192, (4096,), 16), (4096, (4096, 1024, 1024), 16), (30720, (4096,), 16)],
)
def test_one_launch_cluster_sizes(k, widths, rank, numerics):
    """A whole call whose B rows are no more bytes than its A rows runs as one launch with z in
    shared memory, one thread-block cluster of 1, 2, 4 or 8 CTAs per segment (these four
    shapes).  Against the FP32 oracle, and against the same call as two launches (split-K
    shrink into the workspace, then expand), which adds z's K parts in another order."""
    x, a, b, base, slots_t, meta, S, cap = decode_case(k=k, widths=widths, ranks=[rank] * 24, seed=31)
    one = fused(x, a, b, base.clone(), meta, S, numerics=numerics)
    again = fused(x, a, b, base.clone(), meta, S, numerics=numerics)
    assert torch.equal(one, again)  # deterministic
    ws = torch.zeros(workspace_floats(x.shape[0], k, S, cap), dtype=torch.float32, device="cuda")
    two = base.clone()
    sgmv_shrink(x, a, b, two, workspace=ws, **meta, num_slices=S, numerics=numerics)
    sgmv_expand(x, a, b, two, workspace=ws, **meta, num_slices=S, numerics=numerics)
    torch.cuda.synchronize()
    assert np.mean(bf16_bits(one) == bf16_bits(two)) > 0.98
    if numerics == "fp32":
        gate = ref.fp32_gate(values(bf16_bits(one)), fp32_reference(x, a, b, base, slots_t, meta, S))
        assert gate["excess"] <= 1e-2, gate
        assert gate["exact"] > 0.99, gate


def test_reference_numerics_match_decomposed_operators():
    x, a, z, b, _, output, routes, meta = row_case(slices=3, width=4096, columns=1024)
    row_shrink(x, a, z, routes, meta["ranks"], num_slices=3)
    expected = oracle_expand(z, b, output, meta)
    n = output.shape[1]
    out = torch.zeros(output.shape[0], n + 4, dtype=torch.bfloat16, device="cuda")[:, :n]
    out.copy_(output)
    fused(x, a, b, out, meta, 3, numerics="reference")
    got = bf16_bits(out)
    assert rel_l2(values(got), values(expected)) < 0.005
    assert np.mean(got == expected) > 0.95


def test_deterministic_and_graph_replay():
    x, a, b, base, slots_t, meta, S, cap = decode_case(seed=5)
    first = fused(x, a, b, base.clone(), meta, S)
    for _ in range(3):
        again = fused(x, a, b, base.clone(), meta, S)
        assert torch.equal(again, first)
    out = base.clone()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        lora_shrink_expand(x, a, b, out, **meta, num_slices=S)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        lora_shrink_expand(x, a, b, out, **meta, num_slices=S)
    out.copy_(base)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)


def test_rejects_unaligned_output_and_empty_batch():
    x, a, b, base, slots_t, meta, S, cap = decode_case(tokens=8)
    with pytest.raises(ValueError, match="8-byte"):
        lora_shrink_expand(x, a, b, base[:, 1:], **meta, num_slices=S)
    lora_shrink_expand(x[:0], a, b, base[:0], **meta, num_slices=S)


def test_no_device_wait_expired():
    # Every bounded mbarrier wait in the bulk-copy kernels completed in time.
    from loraforge_b200 import _native

    x, a, b, base, slots_t, meta, S, cap = decode_case(seed=9, widths=(14336, 14336))
    fused(x, a, b, base.clone(), meta, S)
    assert _native.device_wait_timeouts(reset=True) == 0
