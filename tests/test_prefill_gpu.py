"""Prefill SGMV (lf_sgmv_prefill: every segment of 1..128 tokens on the tcgen05 tiles, short
ones leaving tile rows idle) on the B200 against the CPU oracle and the decode path."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from cases import values  # noqa: E402
from golden_io import bf16_bits, rel_l2  # noqa: E402
from oracle import cpu_reference as ref  # noqa: E402
from test_fused_gpu import compact_store, fp32_reference  # noqa: E402

from loraforge_b200.ops.fused import lora_shrink_expand, lora_shrink_expand_prefill  # noqa: E402
from loraforge_b200.ops.grouping import group_tokens  # noqa: E402

ROUTING_KEYS = ("segment_indptr", "segment_slots", "token_indices", "segment_count")


def prefill_case(lengths, slots=16, k=1024, widths=(1024,), ranks=None, seed=0, inactive=0.15):
    """Contiguous token runs (one adapter each, some without adapter), like a prefill batch."""
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    ranks = ranks or [64] * slots
    cap = max(ranks)
    S, N, T = len(widths), sum(widths), int(sum(lengths))
    x = torch.randn(T, k, generator=g).bfloat16()
    a = (torch.randn(slots, S * cap, k, generator=g) / k**0.5).bfloat16()
    b, offsets, strides = compact_store(ranks, N, g)
    owners = rng.integers(0, slots, size=len(lengths))
    owners[rng.random(len(lengths)) < inactive] = -1
    ids = np.repeat(owners, lengths).astype(np.int32)
    scales = (torch.rand(slots, generator=g) * 2 + 0.5).float()
    base = (torch.randn(T, N, generator=g) * 0.5).bfloat16()
    dev = "cuda"
    meta = dict(
        b_offsets=torch.tensor(offsets, dtype=torch.int64, device=dev),
        b_strides=torch.tensor(strides, dtype=torch.int32, device=dev),
        ranks=torch.tensor(ranks, dtype=torch.int32, device=dev),
        scales=scales.to(dev),
        slice_offsets=torch.tensor(np.cumsum((0, *widths)), dtype=torch.int32, device=dev),
    )
    slots_t = torch.from_numpy(ids).to(dev)
    return x.to(dev), a.to(dev), b.to(dev), base.to(dev), slots_t, meta, S


def routed(meta, slots_t, num_slots, chunk, runs=False):
    out = dict(meta)
    out.update(zip(ROUTING_KEYS, group_tokens(slots_t, num_slots, chunk=chunk, runs=runs)))
    return out


def geometric(rng, count, mean, total=None):
    lengths = np.maximum(1, rng.geometric(1.0 / mean, size=count))
    if total is not None:
        lengths = np.maximum(1, np.floor(lengths * total / lengths.sum())).astype(np.int64)
        lengths[np.argmax(lengths)] += total - lengths.sum()
    return lengths.astype(np.int64)


def run_prefill(x, a, b, out, meta, S, numerics="fp32"):
    lora_shrink_expand_prefill(x, a, b, out, **meta, num_slices=S, numerics=numerics)
    torch.cuda.synchronize()
    return out


def test_long_and_short_segments_fp32_gate():
    # Geometric run lengths (mean 96, min 1): 128-token tiles, ragged tails, and runs of
    # fewer than 16 tokens that the decode kernels take.
    lengths = geometric(np.random.default_rng(1), 24, 96)
    x, a, b, base, slots_t, meta, S = prefill_case(lengths, k=2048, widths=(1536,), seed=1)
    meta = routed(meta, slots_t, 16, 128)
    out = run_prefill(x, a, b, base.clone(), meta, S)
    expected = fp32_reference(x, a, b, base, slots_t, meta, S)
    gate = ref.fp32_gate(values(bf16_bits(out)), expected)
    assert gate["excess"] <= 1e-2, gate
    assert gate["exact"] > 0.99, gate
    inactive = (slots_t < 0).cpu()
    assert torch.equal(out.cpu()[inactive], base.cpu()[inactive])


@pytest.mark.parametrize("runs", [False, True])
def test_config3_shapes(runs):
    # BASELINE config 3 shapes on a smaller batch: K = N = 5120, rank 64; requests share
    # adapters, so the plain grouping has segments gathered from two runs and the run
    # grouping (the bench's) has none.
    lengths = geometric(np.random.default_rng(2), 16, 256, total=2048)
    x, a, b, base, slots_t, meta, S = prefill_case(lengths, slots=6, k=5120, widths=(5120,), seed=2,
                                                   inactive=0.0)
    meta = routed(meta, slots_t, 6, 128, runs=runs)
    out = run_prefill(x, a, b, base.clone(), meta, S)
    expected = fp32_reference(x, a, b, base, slots_t, meta, S)
    gate = ref.fp32_gate(values(bf16_bits(out)), expected)
    assert gate["excess"] <= 1e-2, gate


def test_mixed_ranks_small_buckets_and_slices():
    ranks = [1, 2, 4, 8, 12, 16, 32, 64] * 2
    lengths = geometric(np.random.default_rng(3), 20, 60)
    x, a, b, base, slots_t, meta, S = prefill_case(
        lengths, k=1024, widths=(768, 256, 256), ranks=ranks, seed=3
    )
    meta = routed(meta, slots_t, len(ranks), 128)
    out = run_prefill(x, a, b, base.clone(), meta, S)
    expected = fp32_reference(x, a, b, base, slots_t, meta, S)
    gate = ref.fp32_gate(values(bf16_bits(out)), expected)
    assert gate["excess"] <= 1e-2, gate


def shifted_store(ranks, n, gen, shifted=()):
    """Compact B with every region 64-element aligned, except that the slots in `shifted`
    start 8 elements later (an offset that is not a whole number of bucket rows)."""
    pieces, offsets, strides, cursor = [], [], [], 0
    for i, r in enumerate(ranks):
        bucket = 1 << (max(1, r) - 1).bit_length()
        pad = (-cursor) % 64 + (8 if i in shifted else 0)
        pieces.append(torch.zeros(pad, dtype=torch.bfloat16))
        cursor += pad
        w = (torch.randn(n, bucket, generator=gen) / max(r, 1) ** 0.5).bfloat16()
        w[:, r:] = 0
        offsets.append(cursor)
        strides.append(bucket)
        pieces.append(w.flatten())
        cursor += w.numel()
    return torch.cat(pieces), offsets, strides


def test_ragged_blocks_and_unaligned_b_offsets():
    # B rows of buckets 16 / 32 / 64 arrive in TMA boxes of 128 and 16 rows plus a cp.async
    # tail.  Slice widths 1000 / 124 / 12 leave partial 256-column blocks: 232 rows (one
    # 128-row box, six 16-row boxes, 8 tail rows), 124 (seven 16-row boxes, 12 tail rows)
    # and 12 (tail rows alone).  Slots 0 and 3 have B offsets that are not a whole number of
    # rows and take the cp.async path for every row.
    ranks = [16, 32, 64, 64, 12, 20, 40, 64]
    widths = (1000, 124, 12)
    lengths = geometric(np.random.default_rng(8), 32, 40)
    x, a, _, base, slots_t, meta, S = prefill_case(
        lengths, slots=len(ranks), k=1024, widths=widths, ranks=ranks, seed=8, inactive=0.05
    )
    assert set(range(len(ranks))) <= set(slots_t.cpu().tolist())
    b, offsets, _ = shifted_store(ranks, sum(widths), torch.Generator().manual_seed(17), shifted={0, 3})
    assert offsets[0] % 16 and offsets[3] % 64 and not offsets[2] % 64
    b = b.cuda()
    meta["b_offsets"] = torch.tensor(offsets, dtype=torch.int64, device="cuda")
    meta = routed(meta, slots_t, len(ranks), 128)
    for numerics in ("fp32", "reference"):
        out = run_prefill(x, a, b, base.clone(), meta, S, numerics)
        if numerics == "fp32":
            expected = fp32_reference(x, a, b, base, slots_t, meta, S)
            gate = ref.fp32_gate(values(bf16_bits(out)), expected)
            assert gate["excess"] <= 1e-2, gate
        else:
            want = base.clone()
            lora_shrink_expand(x, a, b, want, **routed(meta, slots_t, len(ranks), 16), num_slices=S,
                               numerics="reference")
            torch.cuda.synchronize()
            g, w = bf16_bits(out), bf16_bits(want)
            assert rel_l2(values(g), values(w)) < 0.005
            assert np.mean(g == w) > 0.95


def test_batch_under_one_tile_of_tokens():
    # Fewer than 128 tokens: y has no tensor maps and every row is read and written by the
    # epilogue threads themselves.
    lengths = np.array([5, 40, 17, 30, 3], dtype=np.int64)
    x, a, b, base, slots_t, meta, S = prefill_case(lengths, k=1024, widths=(512, 128), seed=9, inactive=0.0)
    meta = routed(meta, slots_t, 16, 128)
    out = run_prefill(x, a, b, base.clone(), meta, S)
    expected = fp32_reference(x, a, b, base, slots_t, meta, S)
    gate = ref.fp32_gate(values(bf16_bits(out)), expected)
    assert gate["excess"] <= 1e-2, gate


def test_reference_numerics_match_decode_path():
    lengths = geometric(np.random.default_rng(4), 16, 80)
    x, a, b, base, slots_t, meta, S = prefill_case(lengths, k=1024, widths=(1024,), seed=4)
    got = run_prefill(x, a, b, base.clone(), routed(meta, slots_t, 16, 128), S, "reference")
    want = base.clone()
    lora_shrink_expand(x, a, b, want, **routed(meta, slots_t, 16, 16), num_slices=S, numerics="reference")
    torch.cuda.synchronize()
    g, w = bf16_bits(got), bf16_bits(want)
    assert rel_l2(values(g), values(w)) < 0.005
    assert np.mean(g == w) > 0.95


def test_deterministic_graph_replay_and_workspace_reuse():
    from loraforge_b200.ops.fused import prefill_workspace_floats

    lengths = geometric(np.random.default_rng(5), 16, 80)
    x, a, b, base, slots_t, meta, S = prefill_case(lengths, k=1024, widths=(1024,), seed=5)
    meta = routed(meta, slots_t, 16, 128)
    ws = torch.zeros(prefill_workspace_floats(x.shape[0], x.shape[1], S, a.shape[1] // S),
                     dtype=torch.float32, device="cuda")
    first = base.clone()
    lora_shrink_expand_prefill(x, a, b, first, **meta, num_slices=S, workspace=ws)
    for _ in range(2):
        again = base.clone()
        lora_shrink_expand_prefill(x, a, b, again, **meta, num_slices=S, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(again, first)
    out = base.clone()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        lora_shrink_expand_prefill(x, a, b, out, **meta, num_slices=S, workspace=ws)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        lora_shrink_expand_prefill(x, a, b, out, **meta, num_slices=S, workspace=ws)
    out.copy_(base)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)


def test_no_device_wait_expired():
    from loraforge_b200 import _native

    lengths = geometric(np.random.default_rng(6), 12, 128)
    x, a, b, base, slots_t, meta, S = prefill_case(lengths, k=2048, widths=(2048,), seed=6)
    run_prefill(x, a, b, base.clone(), routed(meta, slots_t, 16, 128), S)
    assert _native.device_wait_timeouts(reset=True) == 0
