"""Megatron-style tensor-parallel LoRA over B200 ranks (one process per GPU).

The reference runs this path only at tensor parallelism 1 (the fleet backend rejects
TP != 1, src/loraforge/integrations/_sglang_fleet.py:177-178); these helpers add the two
natural shardings of a LoRA-augmented projection:

* column-parallel (QKV, gate/up): rank g owns a 1/G slice of every output slice's
  columns.  A is replicated, so each rank runs the full shrink and expands only its
  columns; there is no communication.
* row-parallel (down): rank g owns a 1/G slice of the input columns of x and A.  Each
  rank's shrink gives a partial z; one all-reduce (sum) of the FP32 z rows
  ([tokens, S*r]) over the group makes it whole, and each rank expands its 1/G slice of
  the output columns (its B rows), so no B row is read twice.

The weight helpers run at load time on either device; the two operators are
asynchronous on the current stream (the all-reduce is the group's collective).
"""

from __future__ import annotations

from loraforge_b200.ops.fused import lora_shrink_expand, sgmv_expand, sgmv_shrink, z_rows


def shard_bounds(width: int, rank: int, world: int) -> tuple[int, int]:
    """[begin, end) of rank's equal share of `width` columns (width % world == 0)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if width % world:
        raise ValueError(f"width {width} is not divisible by {world} ranks")
    share = width // world
    return rank * share, (rank + 1) * share


def shard_a_columns(a, rank: int, world: int):
    """A [slots, S*cap, K] -> rank's input-column shard [slots, S*cap, K/world] (contiguous)."""
    lo, hi = shard_bounds(a.shape[2], rank, world)
    return a[:, :, lo:hi].contiguous()


def shard_b_columns(b, b_offsets, b_strides, slice_widths, rank: int, world: int):
    """Compact B store of rank's output-column shard of every slice.

    b: flat BF16 store; slot g's [N, bucket_g] rows at b_offsets[g] (N = sum of the slice
    widths).  Returns (b_shard, offsets_shard, slice_widths_shard): the slot blocks keep
    their buckets, hold rank's rows of each slice in slice order, and start at 8-element
    boundaries.
    """
    import torch

    offsets = [int(v) for v in b_offsets.tolist()]
    strides = [int(v) for v in b_strides.tolist()]
    n = sum(slice_widths)
    bounds, start = [], 0
    for w in slice_widths:
        lo, hi = shard_bounds(w, rank, world)
        bounds.append((start + lo, start + hi))
        start += w
    pieces, new_offsets, cursor = [], [], 0
    for off, bucket in zip(offsets, strides):
        pad = (-cursor) % 8
        if pad:
            pieces.append(torch.zeros(pad, dtype=b.dtype, device=b.device))
            cursor += pad
        rows = b[off : off + n * bucket].view(n, bucket)
        block = torch.cat([rows[lo:hi] for lo, hi in bounds]).reshape(-1)
        new_offsets.append(cursor)
        pieces.append(block)
        cursor += block.numel()
    shard = torch.cat(pieces) if pieces else b[:0]
    offsets_t = torch.tensor(new_offsets, dtype=torch.int64, device=b_offsets.device)
    return shard, offsets_t, tuple(w // world for w in slice_widths)


def column_parallel(x, a, b_shard, y_shard, **meta) -> None:
    """Column-parallel LoRA: full shrink, expand of this rank's output columns only.

    ``b_shard`` / ``y_shard`` and the routing/metadata keywords as for
    ``lora_shrink_expand`` (``slice_offsets`` of the shard's slice widths).
    """
    lora_shrink_expand(x, a, b_shard, y_shard, **meta)


def row_parallel(x_shard, a_shard, b_shard, y_shard, *, workspace, group=None, **meta) -> None:
    """Row-parallel LoRA: partial shrink, all-reduce of the FP32 z rows, sharded expand.

    ``x_shard`` / ``a_shard`` hold this rank's input columns, ``b_shard`` / ``y_shard``
    its output columns; ``workspace`` (zero-filled before first use) must not be shared
    with another call in flight.  With ``group`` None and no initialised process group
    this is the single-rank computation.
    """
    import torch.distributed as dist

    sgmv_shrink(x_shard, a_shard, b_shard, y_shard, workspace=workspace, **meta)
    num_slices = meta.get("num_slices", 1)
    z = z_rows(workspace, x_shard.shape[0], x_shard.shape[1], num_slices, a_shard.shape[1] // num_slices)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(z, op=dist.ReduceOp.SUM, group=group)
    sgmv_expand(x_shard, a_shard, b_shard, y_shard, workspace=workspace, **meta)
