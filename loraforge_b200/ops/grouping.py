"""Device-side routing metadata: tokens grouped by adapter slot.

Produces the ``segment_indptr / segment_slots / token_indices / segment_count``
tables that ``row_expand`` consumes (src/loraforge/ops/lora_rows.py:115-131) —
the role SGLang's ``prepare_lora_batch`` plays for the reference
(src/loraforge/integrations/_sglang_fleet.py:250-257) — on the GPU, with no host
read of the routing, so the whole routing step can be captured in a CUDA graph.
Grouping is stable: active tokens are ordered by slot, ties by token index.
"""

from __future__ import annotations

from typing import NamedTuple

from loraforge_b200 import _native


class Routing(NamedTuple):
    segment_indptr: object  # int32 [T + 1]
    segment_slots: object  # int32 [T]
    token_indices: object  # int32 [T]
    segment_count: object  # int32 [1]


def empty_routing(num_tokens: int, device) -> Routing:
    """Fixed-address routing buffers for ``num_tokens`` tokens (reuse across replays)."""
    import torch

    n = max(1, num_tokens)
    return Routing(
        torch.zeros(n + 1, dtype=torch.int32, device=device),
        torch.zeros(n, dtype=torch.int32, device=device),
        torch.zeros(n, dtype=torch.int32, device=device),
        torch.zeros(1, dtype=torch.int32, device=device),
    )


def group_tokens(
    slots, num_slots: int, *, chunk: int = 16, runs: bool = False, out: Routing | None = None
) -> Routing:
    """Group tokens by ``slots`` (int32 [T], -1 = no adapter) into <= ``chunk`` token segments.

    ``chunk <= 0`` gives one segment per active slot.  ``runs=True`` groups by runs
    instead (``lf_group_token_runs``): every maximal stretch of consecutive tokens with one
    slot is cut into segments of at most ``chunk`` tokens from its start, in token order,
    and ``token_indices`` lists the active tokens in token order (then the others).  In a
    prefill batch every segment is then one run of a request's tokens, which the prefill
    kernels move as 2-D tiles.  The products are the same either way.  Writes into ``out`` when given (every buffer must have room for T
    tokens), else allocates.
    """
    import torch

    if not isinstance(slots, torch.Tensor):
        raise TypeError("slots must be a torch.Tensor")
    if slots.ndim != 1 or slots.dtype != torch.int32 or not slots.is_contiguous():
        raise ValueError("slots must be a contiguous int32 vector")
    if slots.device.type != "cuda":
        raise ValueError("slots must be on a CUDA device")
    if type(num_slots) is not int or not 1 <= num_slots <= 16384:
        raise ValueError("num_slots must be in 1..16384")
    if type(chunk) is not int:
        raise ValueError("chunk must be an integer")
    T = slots.numel()
    if out is None:
        out = empty_routing(T, slots.device)
    for buf, need in zip(out, (T + 1, T, T, 1)):
        if (
            buf.dtype != torch.int32
            or buf.device != slots.device
            or not buf.is_contiguous()
            or buf.numel() < need
        ):
            raise ValueError("routing buffers must be contiguous int32 with room for every token")
    if type(runs) is not bool:
        raise ValueError("runs must be a bool")
    with torch.cuda.device(slots.device):
        stream = _native.stream_of(slots.device)
        if runs:
            _native.call(
                "lf_group_token_runs",
                slots.data_ptr(),
                T,
                num_slots,
                chunk,
                out.segment_indptr.data_ptr(),
                out.segment_slots.data_ptr(),
                out.token_indices.data_ptr(),
                out.segment_count.data_ptr(),
                stream,
            )
        else:
            _native.call(
                "lf_group_tokens",
                slots.data_ptr(),
                T,
                num_slots,
                chunk,
                out.segment_indptr.data_ptr(),
                out.segment_slots.data_ptr(),
                out.token_indices.data_ptr(),
                out.segment_count.data_ptr(),
                stream,
            )
    return out


def segment_routes(segment_indptr, segment_slots, token_indices, segment_count, num_tokens: int, *, out=None):
    """Per-token slots (int32 [num_tokens], -1 = none) from a segment table.

    The inverse of ``group_tokens``: token ``token_indices[i]`` for ``i`` in segment
    s's range gets ``segment_slots[s]``.  ``segment_count`` (int32, on the device) is
    read by the kernel, so padded tables of captured graphs work unchanged.
    """
    import torch

    for t, name in ((segment_indptr, "segment_indptr"), (segment_slots, "segment_slots"),
                    (token_indices, "token_indices"), (segment_count, "segment_count")):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.ndim != 1 and not (name == "segment_count" and t.ndim == 0):
            raise ValueError(f"{name} must be a vector")
        if t.dtype != torch.int32 or not t.is_contiguous() or t.device != segment_indptr.device:
            raise ValueError(f"{name} must be a contiguous int32 tensor on the routing device")
    if segment_indptr.device.type != "cuda":
        raise ValueError("routing tables must be on a CUDA device")
    if segment_indptr.numel() < segment_slots.numel() + 1:
        raise ValueError("segment_indptr needs one more entry than segment_slots")
    if type(num_tokens) is not int or num_tokens < 0:
        raise ValueError("num_tokens must be a nonnegative integer")
    if out is None:
        out = torch.empty(num_tokens, dtype=torch.int32, device=segment_indptr.device)
    elif out.dtype != torch.int32 or not out.is_contiguous() or out.numel() < num_tokens or out.device != segment_indptr.device:
        raise ValueError("out must be a contiguous int32 buffer with room for every token")
    with torch.cuda.device(segment_indptr.device):
        _native.call(
            "lf_segment_routes", segment_indptr.data_ptr(), segment_slots.data_ptr(),
            token_indices.data_ptr(), segment_count.data_ptr(), segment_slots.numel(),
            token_indices.numel(), num_tokens, out.data_ptr(), _native.stream_of(segment_indptr.device),
        )
    return out[:num_tokens]
