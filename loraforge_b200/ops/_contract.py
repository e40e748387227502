"""Structural argument checks shared by the operators, written as ordered rule lists.

The drop-in contract (src/loraforge/ops/lora_rows.py:54-239 and the BGMV / vLLM modules)
is: look only at tensor metadata (type, rank, dtype, device, shape, strides, data
pointers), never at device values, so a check costs no synchronisation and works while a
CUDA graph is being captured; the first broken rule decides the exception, a TypeError for
a non-tensor and a ValueError for everything else, with the message text callers match.
Each helper here evaluates its rules in a fixed order and raises on the first failure.
"""

from __future__ import annotations

INT32_LIMIT = 2**31


def first_failure(rules) -> None:
    """`rules`: iterable of (broken, message); raise ValueError(message) for the first broken one."""
    for broken, message in rules:
        if broken:
            raise ValueError(message)


def tensor_arg(value, name: str, ndim: int, dtype, device=None) -> None:
    """A CUDA tensor of rank `ndim` and `dtype`, int32-indexable, without autograd history,
    on `device` when one is given."""
    import torch

    if not isinstance(value, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    first_failure((
        (value.ndim != ndim or value.dtype != dtype, f"{name} must be {ndim}D with dtype {dtype}"),
        (max(value.shape, default=0) >= INT32_LIMIT, f"{name} dimensions must fit signed int32 indexing"),
        (value.device.type != "cuda" or (device is not None and value.device != device),
         f"{name} must be on the same CUDA/ROCm GPU"),
        (value.requires_grad, "row operators are inference-only"),
    ))


def vector_arg(value, name: str, dtype, device, length: int | None = None) -> None:
    """A contiguous 1-D `tensor_arg`, of exactly `length` elements when one is given."""
    tensor_arg(value, name, 1, dtype, device)
    first_failure((
        (not value.is_contiguous() or (length is not None and value.numel() != length),
         f"{name} must be contiguous with the required length"),
    ))


def output_is_distinct(output, inputs) -> None:
    """Reject an output whose storage is also an input's storage.

    Whole allocations are compared (not byte ranges), so even disjoint views of one buffer
    count as aliasing: the rule needs no device read and holds for captured graphs, whose
    replays may change what the views contain.
    """
    if not output.numel():
        return
    bases = {t.untyped_storage().data_ptr() for t in inputs if t.numel()}
    first_failure(((output.untyped_storage().data_ptr() in bases,
                    "output must not share storage with an input"),))
