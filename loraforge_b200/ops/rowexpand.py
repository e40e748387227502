"""Fleet-form direct shrink and staged RowExpand on the sm_100a C ABI.

Drop-in for ``loraforge.ops.rowexpand`` (src/loraforge/ops/rowexpand.py:17-92),
the positional form the SGLang fleet backend calls.  Argument checks follow the
reference's C++ ``TORCH_CHECK``s (src/loraforge/ops/csrc/rowexpand.cu:87-125) and
raise ``RuntimeError``; autograd inputs raise ``ValueError`` as in the reference.
Up to four slices; ``row_tile`` 2/4/8/16 only changes the work split.
"""

from __future__ import annotations

from loraforge_b200 import _native
from loraforge_b200.ops.lora_rows import _launch_row_expand, _launch_row_shrink


def rowexpand_extension():
    """Load the native library before any graph capture (the reference's warm-up hook)."""
    return _native.library()


def _check(condition, message="RowExpand argument check failed"):
    if not condition:
        raise RuntimeError(message)


def direct_shrink(x, weights, output, routes, ranks, slices, max_rank):
    """Write live retained A rows; inactive output columns remain unspecified."""
    import torch

    if any(t.requires_grad for t in (x, weights, output)):
        raise ValueError("RowExpand serving operators do not support autograd")
    _check(all(t.is_cuda for t in (x, weights, output, routes, ranks)))
    _check(all(t.dtype == torch.bfloat16 for t in (x, weights, output)))
    _check(
        x.dim() == 2 and weights.dim() == 3 and output.dim() == 2
        and output.shape[0] == x.shape[0]
    )
    _check(
        x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.shape[1] % 8 == 0
        and weights.is_contiguous() and output.is_contiguous()
    )
    _check(
        routes.numel() >= x.shape[0] and routes.dtype == torch.int32
        and ranks.dtype == torch.int32
    )
    _check(
        1 <= slices <= 4 and 1 <= max_rank <= 64 and weights.shape[1] % slices == 0
        and weights.shape[2] == x.shape[1] and output.shape[1] == weights.shape[1]
    )
    _check(
        routes.is_contiguous() and ranks.is_contiguous() and ranks.numel() == weights.shape[0]
    )
    _check(
        all(t.device == x.device for t in (weights, output, routes, ranks)),
        "all tensors must share a device",
    )
    _check(x.data_ptr() % 16 == 0 and weights.data_ptr() % 16 == 0, "unaligned shrink operands")
    _check(weights.shape[1] // slices >= max_rank, "rank capacity below max_rank")
    if x.shape[0] == 0:
        return output
    _launch_row_shrink(x, weights, output, routes, ranks, slices, weights.shape[1] // slices, max_rank)
    return output


def row_expand(
    z,
    store,
    offsets,
    buckets,
    output,
    segments,
    slots,
    permutation,
    ranks,
    scales,
    slice_offsets,
    segment_count,
    capacity,
    *,
    blocks=880,
    threads=256,
    row_tile=16,
):
    """Accumulate the BF16-rounded scaled delta into output on its current stream.

    z uses effective-rank packed slices inside a capacity-strided row; B uses the
    fixed compact regions of a RetainedLayout. No host rank reads, synchronisation
    or allocation happen here.  row_tile 2/4/8 splits each <=16-row segment into
    sub-tiles; 16 keeps whole segments.  Per-token arithmetic is the same for all.
    """
    import torch

    if any(t.requires_grad for t in (z, store, output, scales)):
        raise ValueError("RowExpand serving operators do not support autograd")
    tensors = (z, store, output, offsets, buckets, segments, slots, permutation, ranks,
               scales, slice_offsets, segment_count)
    _check(all(t.is_cuda for t in tensors))
    _check(
        z.dtype == store.dtype == output.dtype == torch.bfloat16 and scales.dtype == torch.float32
    )
    n = output.shape[1] if output.dim() == 2 else 0
    _check(
        z.is_contiguous() and store.is_contiguous() and output.stride(1) == 1
        and 2 <= slice_offsets.numel() <= 5 and blocks > 0 and threads in (128, 256)
    )
    _check(
        all(t.dtype == torch.int32 for t in (ranks, buckets, segments, slots, permutation,
                                              slice_offsets, segment_count))
        and offsets.dtype == torch.int64
    )
    _check(z.dim() == 2 and store.dim() == 1 and output.dim() == 2 and n > 0 and capacity > 0)
    _check(
        output.shape[0] == z.shape[0]
        and z.shape[1] == capacity * (slice_offsets.numel() - 1)
    )
    _check(segment_count.numel() == 1)
    _check(
        buckets.numel() == ranks.numel() == offsets.numel() == scales.numel()
    )
    _check(segments.numel() >= slots.numel() + 1 and permutation.numel() >= z.shape[0])
    _check(output.stride(0) >= n and store.data_ptr() % 16 == 0)
    _check(all(t.device == z.device for t in tensors), "all tensors must share a device")
    _check(
        all(t.is_contiguous() for t in tensors[3:]), "metadata must be contiguous"
    )
    _check(row_tile in (2, 4, 8, 16), "row_tile must be 2, 4, 8, or 16")
    _check(blocks <= 65535, "blocks must be in 1..65535")
    if z.shape[0] == 0:
        return output
    with torch.cuda.device(z.device):
        _launch_row_expand(
            z, store, offsets, buckets, output, segments, slots, permutation, ranks,
            scales, slice_offsets, segment_count, capacity, blocks, threads, row_tile,
        )
    return output
