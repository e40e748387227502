"""Prefill SGMV (lf_sgmv_prefill: tcgen05 tiles for segments of 16..128 tokens, decode
kernels for shorter ones) on the B200 against the CPU oracle and the decode path."""

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


def routed(meta, slots_t, num_slots, chunk):
    out = dict(meta)
    out.update(zip(ROUTING_KEYS, group_tokens(slots_t, num_slots, chunk=chunk)))
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


def test_config3_shapes():
    # BASELINE config 3 shapes on a smaller batch: K = N = 5120, rank 64.
    lengths = geometric(np.random.default_rng(2), 8, 256, total=1024)
    x, a, b, base, slots_t, meta, S = prefill_case(lengths, k=5120, widths=(5120,), seed=2, inactive=0.0)
    meta = routed(meta, slots_t, 16, 128)
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
