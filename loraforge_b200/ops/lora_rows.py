"""Retained-rank row operators (``row_shrink`` / ``row_expand``) over the sm_100a C ABI.

These keep the public surface of ``loraforge.ops.lora_rows``
(src/loraforge/ops/lora_rows.py:54-239): the call signatures and keyword names, the
order in which arguments are checked, and the exception types and message texts.  The
checks read tensor metadata only, so a call never waits for the GPU and a warmed call can
be recorded into a CUDA graph.  The work runs in ``lf_row_shrink`` (one warp per token and
rank row, summed in the reference kernel's order, so z matches it bit for bit) and
``lf_row_expand`` (the reference's element arithmetic, so equal inputs give equal bits).
"""

from __future__ import annotations

from typing import TYPE_CHECKING

from loraforge_b200 import _native
from loraforge_b200.annotations import ExperimentalAPI
from loraforge_b200.ops._contract import first_failure, output_is_distinct, tensor_arg, vector_arg

if TYPE_CHECKING:
    from torch import Tensor

# Retained-rank limits of the operator pair.
MAX_SLICES = 3
MAX_RANK = 64


@ExperimentalAPI(
    reason="BF16 retained-rank inference operator; sm_100a CUDA, caller-owned device metadata."
)
def row_shrink(
    x: Tensor,
    a: Tensor,
    output: Tensor,
    slots: Tensor,
    ranks: Tensor,
    *,
    num_slices: int = 1,
    max_rank: int = 64,
) -> None:
    """z[t] = A[slots[t]] @ x[t] for the live rank rows only, written into ``output``.

    Shapes: x [T, K]; a [num_slots, num_slices * capacity, K]; output
    [T, num_slices * capacity].  A slot of rank r keeps slice s's r rows at rows
    s*r .. s*r + r - 1 of its A block, and the results go to the same columns of its
    output row, each an FP32 sum rounded once to BF16.  Columns beyond num_slices * r,
    tokens routed to slot -1 and slots of rank 0 are not written.  Every live rank must
    be at most ``max_rank``; K and x's row stride must be multiples of 8 elements.
    """
    import torch

    tensor_arg(x, "x", 2, torch.bfloat16)
    tensor_arg(a, "a", 3, torch.bfloat16, x.device)
    tensor_arg(output, "output", 2, torch.bfloat16, x.device)
    _int_in_range(num_slices, 1, MAX_SLICES, "num_slices must be in 1..3")
    _int_in_range(max_rank, 1, MAX_RANK, "max_rank must be in 1..64")
    slots_total, rows, width = a.shape
    first_failure((
        (slots_total < 1 or rows % num_slices or rows // num_slices < max_rank or width != x.shape[1]
         or tuple(output.shape) != (x.shape[0], rows),
         "A/output shapes must agree with slices and rank capacity"),
        (not _rows_aligned(x) or a.data_ptr() % 16 or not a.is_contiguous() or not output.is_contiguous(),
         "expected aligned A/x and contiguous A/output"),
    ))
    vector_arg(slots, "slots", torch.int32, x.device, x.shape[0])
    vector_arg(ranks, "ranks", torch.int32, x.device, slots_total)
    output_is_distinct(output, (x, a, slots, ranks))
    if x.shape[0]:
        _launch_row_shrink(x, a, output, slots, ranks, num_slices, rows // num_slices, max_rank)


def _int_in_range(value, lo, hi, message) -> None:
    first_failure(((type(value) is not int or not lo <= value <= hi, message),))


def _rows_aligned(x) -> bool:
    """BF16 rows of a multiple of 8 elements, unit column stride, 16-byte aligned start."""
    width, stride = x.shape[1], x.stride(0)
    return (width >= 1 and width % 8 == 0 and x.stride(1) == 1 and stride >= width
            and stride % 8 == 0 and x.data_ptr() % 16 == 0)


def _launch_row_shrink(x, a, output, slots, ranks, num_slices, capacity, max_rank):
    import torch

    with torch.cuda.device(x.device):
        _native.call(
            "lf_row_shrink", x.data_ptr(), x.stride(0), a.data_ptr(), output.data_ptr(),
            slots.data_ptr(), ranks.data_ptr(), x.shape[0], x.shape[1], a.shape[0], num_slices,
            capacity, max_rank, _native.stream_of(x.device),
        )


@ExperimentalAPI(
    reason="Compact-B RowExpand; sm_100a CUDA, fixed-address metadata/lifetime contract."
)
def row_expand(
    z: Tensor,
    b: Tensor,
    output: Tensor,
    *,
    b_offsets: Tensor,
    b_strides: Tensor,
    ranks: Tensor,
    scales: Tensor,
    segment_indptr: Tensor,
    segment_slots: Tensor,
    token_indices: Tensor,
    slice_offsets: Tensor,
    segment_count: Tensor,
    blocks: int | None = None,
    threads: int = 256,
) -> None:
    """output[t, cols of slice s] += BF16(scale_g * B_g[cols, :r] @ z[t, s*r : s*r + r]).

    Routing: segment i covers positions segment_indptr[i] .. segment_indptr[i+1] - 1 of
    ``token_indices`` (at most 16 tokens, each in one live segment only), all of slot
    segment_slots[i]; ``segment_count`` (int32 on the device) says how many segments are
    live, so a captured graph replays with new routes.  B is one flat BF16 store: slot g's
    [N, b_strides[g]] block starts b_offsets[g] elements in, b_strides[g] a power of two
    in 1..64 and at least the slot's rank, zero beyond it.  ``slice_offsets`` splits the
    N output columns into the slices.

    Each product is an FP32 dot product; it is scaled, rounded to BF16, added to the BF16
    output and rounded again.  Segments of slot -1 or rank 0 change nothing.  The caller
    owns every buffer's lifetime and the ordering of metadata writes on the stream.
    """
    import torch

    tensor_arg(z, "z", 2, torch.bfloat16)
    tensor_arg(b, "b", 1, torch.bfloat16, z.device)
    tensor_arg(output, "output", 2, torch.bfloat16, z.device)
    vector_arg(ranks, "ranks", torch.int32, z.device)
    nslots = ranks.numel()
    per_slot = (("b_offsets", b_offsets, torch.int64), ("b_strides", b_strides, torch.int32),
                ("scales", scales, torch.float32))
    for name, tensor, dtype in per_slot:
        vector_arg(tensor, name, dtype, z.device, nslots)
    vector_arg(segment_slots, "segment_slots", torch.int32, z.device)
    vector_arg(segment_indptr, "segment_indptr", torch.int32, z.device, segment_slots.numel() + 1)
    vector_arg(token_indices, "token_indices", torch.int32, z.device)
    vector_arg(slice_offsets, "slice_offsets", torch.int32, z.device)
    vector_arg(segment_count, "segment_count", torch.int32, z.device, 1)
    slices = slice_offsets.numel() - 1
    first_failure((
        (nslots < 1 or not 1 <= slices <= MAX_SLICES or z.shape[1] < slices or z.shape[1] % slices
         or output.shape[0] != z.shape[0] or output.shape[1] < 1,
         "invalid slots, slice count or activation/output shape"),
        (not z.is_contiguous() or not b.is_contiguous() or b.data_ptr() % 16 or output.stride(1) != 1
         or output.stride(0) < output.shape[1],
         "expected contiguous z/aligned B and nonoverlapping output rows"),
        (blocks is not None and (type(blocks) is not int or not 1 <= blocks <= 65535),
         "blocks must be in 1..65535"),
        (type(threads) is not int or threads not in (128, 256), "threads must be 128 or 256"),
    ))
    first_failure(((segment_slots.numel() * -(-output.shape[1] // threads) >= 2**31,
                    "segment work count must fit signed int32 indexing"),))
    output_is_distinct(output, (z, b, b_offsets, b_strides, ranks, scales, segment_indptr,
                                segment_slots, token_indices, slice_offsets, segment_count))
    if not z.shape[0]:
        return
    with torch.cuda.device(z.device):
        if blocks is None:  # 0: the kernel's own resident-CTA count times the SMs
            blocks = 0
        _launch_row_expand(
            z, b, b_offsets, b_strides, output, segment_indptr, segment_slots,
            token_indices, ranks, scales, slice_offsets, segment_count,
            z.shape[1] // slices, blocks, threads, 16,
        )


def _launch_row_expand(
    z, b, b_offsets, b_strides, output, segment_indptr, segment_slots, token_indices,
    ranks, scales, slice_offsets, segment_count, capacity, blocks, threads, row_tile,
):
    _native.call(
        "lf_row_expand", z.data_ptr(), b.data_ptr(), b_offsets.data_ptr(), b_strides.data_ptr(),
        output.data_ptr(), output.stride(0), segment_indptr.data_ptr(), segment_slots.data_ptr(),
        token_indices.data_ptr(), ranks.data_ptr(), scales.data_ptr(), slice_offsets.data_ptr(),
        segment_count.data_ptr(), z.shape[0], output.shape[1], slice_offsets.numel() - 1, capacity,
        ranks.numel(), segment_slots.numel(), blocks, threads, row_tile, _native.stream_of(z.device),
    )
