"""Tensor-parallel LoRA kernels on one B200: two ranks' shards computed on the same
device (the all-reduce of the row-parallel z done by hand) against the unsharded
fused operator and the FP32 oracle."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from cases import values  # noqa: E402
from golden_io import bf16_bits  # noqa: E402
from oracle import cpu_reference as ref  # noqa: E402
from test_fused_gpu import decode_case, fp32_reference  # noqa: E402

from loraforge_b200.ops.fused import (  # noqa: E402
    lora_shrink_expand,
    sgmv_expand,
    sgmv_shrink,
    workspace_floats,
    z_rows,
)
from loraforge_b200.ops.sharded import (  # noqa: E402
    column_parallel,
    shard_a_columns,
    shard_b_columns,
    shard_bounds,
)

WORLD = 2


def shard_meta(meta, b_offsets, widths):
    m = dict(meta)
    m["b_offsets"] = b_offsets
    m["slice_offsets"] = torch.tensor(np.cumsum((0, *widths)), dtype=torch.int32, device="cuda")
    return m


def test_column_parallel_matches_unsharded_bitwise():
    widths = (2048, 2048)
    x, a, b, base, slots_t, meta, S, cap = decode_case(tokens=96, slots=16, k=2048, widths=widths,
                                                      ranks=[32] * 16, seed=11)
    full = base.clone()
    lora_shrink_expand(x, a, b, full, **meta, num_slices=S)
    for r in range(WORLD):
        bs, offs, sw = shard_b_columns(b, meta["b_offsets"], meta["b_strides"], widths, r, WORLD)
        cols = [c for s, w in enumerate(widths) for c in range(sum(widths[:s]) + shard_bounds(w, r, WORLD)[0],
                                                                  sum(widths[:s]) + shard_bounds(w, r, WORLD)[1])]
        y = base[:, cols].contiguous()
        column_parallel(x, a, bs, y, **shard_meta(meta, offs, sw), num_slices=S)
        torch.cuda.synchronize()
        assert torch.equal(y, full[:, cols])


def test_row_parallel_two_shards_with_z_sum():
    widths = (2048,)
    x, a, b, base, slots_t, meta, S, cap = decode_case(tokens=96, slots=16, k=4096, widths=widths,
                                                      ranks=[32] * 16, seed=12)
    expected = fp32_reference(x, a, b, base, slots_t, meta, S)
    T = x.shape[0]
    shards = []
    for r in range(WORLD):
        xs = x[:, slice(*shard_bounds(x.shape[1], r, WORLD))].contiguous()
        As = shard_a_columns(a, r, WORLD)
        bs, offs, sw = shard_b_columns(b, meta["b_offsets"], meta["b_strides"], widths, r, WORLD)
        ys = base[:, slice(*shard_bounds(widths[0], r, WORLD))].contiguous()
        ws = torch.zeros(workspace_floats(T, xs.shape[1], S, cap), dtype=torch.float32, device="cuda")
        m = shard_meta(meta, offs, sw)
        sgmv_shrink(xs, As, bs, ys, workspace=ws, **m, num_slices=S)
        shards.append((xs, As, bs, ys, ws, m))
    # The all-reduce of the z rows, done on one device.
    zs = [z_rows(ws, T, xs.shape[1], S, cap) for xs, _, _, _, ws, _ in shards]
    total = zs[0] + zs[1]
    for z in zs:
        z.copy_(total)
    for xs, As, bs, ys, ws, m in shards:
        sgmv_expand(xs, As, bs, ys, workspace=ws, **m, num_slices=S)
    torch.cuda.synchronize()
    got = torch.cat([s[3] for s in shards], dim=1)
    gate = ref.fp32_gate(values(bf16_bits(got)), expected)
    assert gate["excess"] <= 1e-2, gate


def test_split_halves_agree_with_fused_call():
    """The two halves (shrink, then expand on the same workspace; the row-parallel path) compute
    what one fused call computes.  The fused call runs the one-launch kernel, which adds z's K
    parts in another order, so the two agree within the FP32 gate and on almost every output
    bit rather than bit for bit; each is deterministic."""
    x, a, b, base, slots_t, meta, S, cap = decode_case(tokens=64, slots=12, seed=13)
    expected = fp32_reference(x, a, b, base, slots_t, meta, S)
    outs = []
    for _ in range(2):
        fused = base.clone()
        lora_shrink_expand(x, a, b, fused, **meta, num_slices=S)
        ws = torch.zeros(workspace_floats(x.shape[0], x.shape[1], S, cap), dtype=torch.float32, device="cuda")
        split = base.clone()
        sgmv_shrink(x, a, b, split, workspace=ws, **meta, num_slices=S)
        sgmv_expand(x, a, b, split, workspace=ws, **meta, num_slices=S)
        torch.cuda.synchronize()
        outs.append((fused, split))
    (fused, split), (fused2, split2) = outs
    assert torch.equal(fused, fused2) and torch.equal(split, split2)
    for out in (fused, split):
        gate = ref.fp32_gate(values(bf16_bits(out)), expected)
        assert gate["excess"] <= 1e-2, gate
    assert np.mean(bf16_bits(split) == bf16_bits(fused)) > 0.99
