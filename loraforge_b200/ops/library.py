"""``torch.library`` registrations of the operators, for graph capture and ``torch.compile``.

The operators mutate a caller-owned output and return nothing, and their argument checks
read tensor metadata only; as custom ops with declared mutations they are opaque nodes
to ``torch.compile`` (no tracing into ctypes, no graph break) and record into CUDA graphs
like any other kernel launch.  The pattern follows the reference's vLLM op
(src/loraforge/integrations/vllm.py:24).  ``register()`` is idempotent and returns the
op handles; after it, the ops are also reachable as ``torch.ops.loraforge_b200.<name>``.

    ops = register()
    ops.row_shrink(x, a, z, slots, ranks, 1, 64)
    ops.row_expand(z, b, y, b_offsets, b_strides, ranks, scales, segment_indptr,
                   segment_slots, token_indices, slice_offsets, segment_count, None, 256)
    ops.lora_shrink_expand(x, a, b, y, b_offsets, b_strides, ranks, scales, segment_indptr,
                           segment_slots, token_indices, slice_offsets, segment_count,
                           num_slices, "fp32", workspace)
"""

from functools import lru_cache
from types import SimpleNamespace
from typing import Optional


@lru_cache(maxsize=1)
def register() -> SimpleNamespace:
    import torch

    from loraforge_b200.ops.fused import lora_shrink_expand as _fused
    from loraforge_b200.ops.lora_rows import row_expand as _expand
    from loraforge_b200.ops.lora_rows import row_shrink as _shrink

    Tensor = torch.Tensor  # annotations are evaluated when the ops are defined

    @torch.library.custom_op("loraforge_b200::row_shrink", mutates_args=("output",))
    def row_shrink(x: Tensor, a: Tensor, output: Tensor, slots: Tensor, ranks: Tensor,
                   num_slices: int, max_rank: int) -> None:
        _shrink(x, a, output, slots, ranks, num_slices=num_slices, max_rank=max_rank)

    @torch.library.custom_op("loraforge_b200::row_expand", mutates_args=("output",))
    def row_expand(z: Tensor, b: Tensor, output: Tensor, b_offsets: Tensor, b_strides: Tensor,
                   ranks: Tensor, scales: Tensor, segment_indptr: Tensor, segment_slots: Tensor,
                   token_indices: Tensor, slice_offsets: Tensor, segment_count: Tensor,
                   blocks: Optional[int], threads: int) -> None:
        _expand(z, b, output, b_offsets=b_offsets, b_strides=b_strides, ranks=ranks, scales=scales,
                segment_indptr=segment_indptr, segment_slots=segment_slots, token_indices=token_indices,
                slice_offsets=slice_offsets, segment_count=segment_count, blocks=blocks, threads=threads)

    @torch.library.custom_op("loraforge_b200::lora_shrink_expand", mutates_args=("output", "workspace"))
    def lora_shrink_expand(x: Tensor, a: Tensor, b: Tensor, output: Tensor, b_offsets: Tensor,
                           b_strides: Tensor, ranks: Tensor, scales: Tensor, segment_indptr: Tensor,
                           segment_slots: Tensor, token_indices: Tensor, slice_offsets: Tensor,
                           segment_count: Tensor, num_slices: int, numerics: str,
                           workspace: Optional[Tensor]) -> None:
        _fused(x, a, b, output, b_offsets=b_offsets, b_strides=b_strides, ranks=ranks, scales=scales,
               segment_indptr=segment_indptr, segment_slots=segment_slots, token_indices=token_indices,
               slice_offsets=slice_offsets, segment_count=segment_count, num_slices=num_slices,
               numerics=numerics, workspace=workspace)

    # Mutations only: the abstract (fake) implementations produce nothing.
    for op in (row_shrink, row_expand, lora_shrink_expand):
        op.register_fake(lambda *args, **kwargs: None)
    return SimpleNamespace(row_shrink=row_shrink, row_expand=row_expand,
                           lora_shrink_expand=lora_shrink_expand)
