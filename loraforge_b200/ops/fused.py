"""Grouped retained-rank shrink -> expand for decode segments (SGMV, z kept in FP32).

``lora_shrink_expand`` takes the operands of ``row_shrink`` (x, packed A) and of
``row_expand`` (compact B store, per-slot metadata, routing tables) and computes
``output += scale * B @ (A @ x)`` for every routed token in one call: a persistent
grouped shrink kernel (each adapter's A rows streamed once per segment, K split into
chunks whose partial sums are reduced deterministically) chained by programmatic
dependent launch to a persistent grouped expand kernel, both fed by bulk-copy
pipelines, with the rank-r intermediate kept in FP32.  It is the B200 form of the
reference's two-kernel decode path (src/loraforge/ops/lora_rows.py:54-239 as driven
by src/loraforge/integrations/_sglang_fleet.py:271-407).

``numerics="fp32"`` (default) keeps z in FP32 and rounds the output once;
``numerics="reference"`` reproduces the retained-rank operators' contract (BF16 z,
BF16-rounded scaled delta, BF16 sum), so it agrees with ``row_shrink`` followed by
``row_expand`` up to the FP32 summation order of the shrink.
"""

from __future__ import annotations

from loraforge_b200 import _native
from loraforge_b200.annotations import ExperimentalAPI
from loraforge_b200.ops._contract import output_is_distinct, tensor_arg, vector_arg

NUMERICS = {"fp32": 0, "reference": 1}


def workspace_floats(tokens: int, width: int, num_slices: int, capacity: int) -> int:
    """Elements of the FP32 workspace ``lora_shrink_expand`` needs for these sizes."""
    return _native.fused_workspace_floats(tokens, width, num_slices, capacity)


@ExperimentalAPI(reason="Fused BF16 decode shrink/expand; sm_100a tensor cores, caller-owned metadata.")
def lora_shrink_expand(
    x,
    a,
    b,
    output,
    *,
    b_offsets,
    b_strides,
    ranks,
    scales,
    segment_indptr,
    segment_slots,
    token_indices,
    slice_offsets,
    segment_count,
    num_slices: int = 1,
    numerics: str = "fp32",
    workspace=None,
) -> None:
    """Add ``scale * B_g @ (A_g @ x[t])`` to ``output[t]`` for every routed token.

    x [tokens, width]; A [slots, slices*capacity, width]; output [tokens, N] with
    slice_offsets partitioning N; B flat with b_offsets (8-element aligned) and
    power-of-two b_strides in 1..64; segments of at most 16 tokens, one slot each
    (``group_tokens(..., chunk=16)``).  Slot -1 / rank-0 segments leave output
    unchanged.  ``workspace`` is an optional FP32 buffer of at least
    ``workspace_floats(tokens, width, num_slices, capacity)`` elements for the
    shrink's partial sums, the FP32 z rows and per-segment completion counters
    (allocated per call when omitted; pass one to keep a captured graph
    allocation-free).  A caller-owned workspace must be zero-filled before its
    first use (``torch.zeros``); every call leaves its counters at zero again, so
    one workspace serves any sequence of calls of the same sizes on one stream.
    ``workspace="builtin"`` uses the library's fixed per-device scratch instead
    (``lf_fused_shrink_expand_noalloc``: up to 16384 tokens, any sequence of sizes,
    no allocation; the first call on a device should come before any stream
    capture); calls that use it must not run concurrently on different streams of
    one device.
    """
    _launch(
        "lf_fused_shrink_expand", _native.fused_workspace_floats, x, a, b, output, b_offsets,
        b_strides, ranks, scales, segment_indptr, segment_slots, token_indices, slice_offsets,
        segment_count, num_slices, numerics, workspace,
    )


def reset_workspace(workspace, tokens: int, width: int, num_slices: int, capacity: int) -> None:
    """Zero the completion counters of a ``lora_shrink_expand`` workspace (on its stream).

    Every call leaves them at zero, also after a bounded device wait ran out (the kernel
    counts the units it gave up on); use this when a workspace's contents may have been
    overwritten, before reusing it.  Asynchronous; allocates nothing.
    """
    import torch

    need = workspace_floats(tokens, width, num_slices, capacity)
    if not isinstance(workspace, torch.Tensor) or workspace.dtype != torch.float32 or workspace.numel() < need:
        raise ValueError(f"workspace must be an FP32 tensor of >= {need} elements")
    with torch.cuda.device(workspace.device):
        _native.call("lf_fused_workspace_reset", workspace.data_ptr(), workspace.numel(), tokens, width,
                     num_slices, capacity, _native.stream_of(workspace.device))


def reset_builtin_workspace(device=None) -> None:
    """Zero the counters of the library's built-in scratch (``workspace="builtin"``) on
    ``device`` (default: the current device), on its current stream.  Allocates nothing."""
    import torch

    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(device):
        _native.call("lf_fused_noalloc_reset", _native.stream_of(device))


def prefill_workspace_floats(tokens: int, width: int, num_slices: int, capacity: int) -> int:
    """Elements of the FP32 workspace ``lora_shrink_expand_prefill`` needs for these sizes."""
    return _native.prefill_workspace_floats(tokens, width, num_slices, capacity)


@ExperimentalAPI(reason="Fused BF16 prefill shrink/expand; sm_100a tcgen05 tensor cores, caller-owned metadata.")
def lora_shrink_expand_prefill(
    x,
    a,
    b,
    output,
    *,
    b_offsets,
    b_strides,
    ranks,
    scales,
    segment_indptr,
    segment_slots,
    token_indices,
    slice_offsets,
    segment_count,
    num_slices: int = 1,
    numerics: str = "fp32",
    workspace=None,
) -> None:
    """``lora_shrink_expand`` for prefill batches: segments of up to 128 tokens.

    Route with ``group_tokens(..., chunk=128, runs=True)``: segments that are one run of
    tokens move their y rows as 2-D TMA tiles; segments gathered from several runs (a
    plain ``chunk=128`` grouping, or a serving framework's chunks) are correct too, with
    their y rows copied row by row.  Every segment runs on the tcgen05 tensor cores
    (128-token tiles, FP32 accumulators in TMEM; a short segment leaves tile rows idle but
    moves no extra x or y bytes).  Same operands, numerics and workspace rules
    as ``lora_shrink_expand`` with ``prefill_workspace_floats`` for the size.  The B200
    form of the reference's prefill SGMV (the rank-aware shrink,
    src/loraforge/integrations/_sglang_rank_aware.py:14-171, and the chunked expand it
    pairs with, src/loraforge/integrations/_sglang_fleet.py:310-313).
    """
    _launch(
        "lf_sgmv_prefill", _native.prefill_workspace_floats, x, a, b, output, b_offsets,
        b_strides, ranks, scales, segment_indptr, segment_slots, token_indices, slice_offsets,
        segment_count, num_slices, numerics, workspace,
    )


def _launch(entry, sizer, x, a, b, output, b_offsets, b_strides, ranks, scales,
            segment_indptr, segment_slots, token_indices, slice_offsets, segment_count,
            num_slices, numerics, workspace):
    import torch

    _check_operands(x, a, b, output, b_offsets, b_strides, ranks, scales, segment_indptr, segment_slots,
                    token_indices, slice_offsets, segment_count, num_slices, numerics)
    nslots = ranks.numel()
    capacity = a.shape[1] // num_slices
    if isinstance(workspace, str):
        if workspace != "builtin" or entry != "lf_fused_shrink_expand":
            raise ValueError("workspace='builtin' applies to lora_shrink_expand only")
        if x.shape[0] == 0:
            return
        with torch.cuda.device(x.device):
            _native.call(
                "lf_fused_shrink_expand_noalloc", x.data_ptr(), x.stride(0), a.data_ptr(),
                b.data_ptr(), b_offsets.data_ptr(), b_strides.data_ptr(), output.data_ptr(),
                output.stride(0), segment_indptr.data_ptr(), segment_slots.data_ptr(),
                token_indices.data_ptr(), ranks.data_ptr(), scales.data_ptr(),
                slice_offsets.data_ptr(), segment_count.data_ptr(), x.shape[0], x.shape[1],
                output.shape[1], num_slices, capacity, nslots, segment_slots.numel(),
                NUMERICS[numerics], _native.stream_of(x.device),
            )
        return
    need = sizer(x.shape[0], x.shape[1], num_slices, capacity)
    if workspace is None:
        workspace = torch.zeros(need, dtype=torch.float32, device=x.device)
    if (
        not isinstance(workspace, torch.Tensor)
        or workspace.dtype != torch.float32
        or workspace.device != x.device
        or not workspace.is_contiguous()
        or workspace.numel() < need
        or workspace.data_ptr() % 16
    ):
        raise ValueError(
            f"workspace must be a contiguous 16-byte aligned FP32 buffer of >= {need} "
            f"elements on the same device ({sizer.__name__})"
        )
    if x.shape[0] == 0:
        return
    with torch.cuda.device(x.device):
        _native.call(
            entry,
            x.data_ptr(),
            x.stride(0),
            a.data_ptr(),
            b.data_ptr(),
            b_offsets.data_ptr(),
            b_strides.data_ptr(),
            output.data_ptr(),
            output.stride(0),
            segment_indptr.data_ptr(),
            segment_slots.data_ptr(),
            token_indices.data_ptr(),
            ranks.data_ptr(),
            scales.data_ptr(),
            slice_offsets.data_ptr(),
            segment_count.data_ptr(),
            workspace.data_ptr(),
            workspace.numel(),
            x.shape[0],
            x.shape[1],
            output.shape[1],
            num_slices,
            capacity,
            nslots,
            segment_slots.numel(),
            NUMERICS[numerics],
            _native.stream_of(x.device),
        )


def _check_operands(x, a, b, output, b_offsets, b_strides, ranks, scales, segment_indptr, segment_slots,
                    token_indices, slice_offsets, segment_count, num_slices, numerics):
    """Structural checks of the fused operators' operands and routing (no device reads)."""
    import torch

    tensor_arg(x, "x", 2, torch.bfloat16)
    tensor_arg(a, "a", 3, torch.bfloat16, x.device)
    tensor_arg(b, "b", 1, torch.bfloat16, x.device)
    tensor_arg(output, "output", 2, torch.bfloat16, x.device)
    if type(num_slices) is not int or not 1 <= num_slices <= 4:
        raise ValueError("num_slices must be in 1..4")
    if numerics not in NUMERICS:
        raise ValueError("numerics must be 'fp32' or 'reference'")
    vector_arg(ranks, "ranks", torch.int32, x.device, a.shape[0])
    nslots = ranks.numel()
    for tensor, name, dtype in (
        (b_offsets, "b_offsets", torch.int64),
        (b_strides, "b_strides", torch.int32),
        (scales, "scales", torch.float32),
    ):
        vector_arg(tensor, name, dtype, x.device, nslots)
    vector_arg(segment_slots, "segment_slots", torch.int32, x.device)
    vector_arg(segment_indptr, "segment_indptr", torch.int32, x.device, segment_slots.numel() + 1)
    vector_arg(token_indices, "token_indices", torch.int32, x.device)
    vector_arg(slice_offsets, "slice_offsets", torch.int32, x.device, num_slices + 1)
    vector_arg(segment_count, "segment_count", torch.int32, x.device, 1)
    if (
        a.shape[1] % num_slices
        or a.shape[2] != x.shape[1]
        or output.shape[0] != x.shape[0]
        or output.shape[1] < 1
    ):
        raise ValueError("A/output shapes must agree with slices and tokens")
    if (
        x.shape[1] % 8
        or x.stride(1) != 1
        or x.stride(0) % 8
        or x.stride(0) < x.shape[1]
        or x.data_ptr() % 16
        or not a.is_contiguous()
        or a.data_ptr() % 16
        or not b.is_contiguous()
        or b.data_ptr() % 16
    ):
        raise ValueError("expected aligned A/B/x with width and row stride multiples of 8")
    if output.stride(1) != 1 or output.stride(0) % 4 or output.stride(0) < output.shape[1] or output.data_ptr() % 8:
        raise ValueError("output rows must be 8-byte aligned with a row stride multiple of 4")
    output_is_distinct(
        output,
        (x, a, b, b_offsets, b_strides, ranks, scales, segment_indptr, segment_slots,
         token_indices, slice_offsets, segment_count),
    )


def sgmv_shrink(x, a, b, output, *, workspace, **routing) -> None:
    """First half of ``lora_shrink_expand``: z = A_g @ x[t] into ``workspace``.

    Same keyword arguments as ``lora_shrink_expand`` (``output`` and B are validated
    but not touched).  The FP32 z rows stay in ``workspace`` (see ``z_rows``) until
    ``sgmv_expand`` consumes them; pass the same workspace and sizes to both.
    """
    if workspace is None:
        raise ValueError("sgmv_shrink needs a caller-owned workspace that outlives the call")
    _launch_routed("lf_sgmv_shrink", x, a, b, output, workspace, routing)


def sgmv_expand(x, a, b, output, *, workspace, **routing) -> None:
    """Second half of ``lora_shrink_expand``: output += scale * B_g @ z from ``workspace``."""
    if workspace is None:
        raise ValueError("sgmv_expand needs the workspace sgmv_shrink wrote")
    _launch_routed("lf_sgmv_expand", x, a, b, output, workspace, routing)


def z_rows(workspace, tokens: int, width: int, num_slices: int, capacity: int):
    """View of the FP32 z rows ``sgmv_shrink`` leaves in ``workspace``: [tokens, row].

    Row t belongs to the token at position t of ``token_indices``; columns s*r + k hold
    slice s, rank index k.  Summing this view over the ranks of a row-parallel
    projection (A columns sharded) between ``sgmv_shrink`` and ``sgmv_expand`` gives
    every rank the full z.
    """
    offset, row = _native.fused_z_rows(tokens, width, num_slices, capacity)
    return workspace[offset : offset + max(tokens, 1) * row].view(max(tokens, 1), row)[:tokens]


def _launch_routed(entry, x, a, b, output, workspace, routing):
    routing = dict(routing)
    num_slices = routing.pop("num_slices", 1)
    numerics = routing.pop("numerics", "fp32")
    keys = ("b_offsets", "b_strides", "ranks", "scales", "segment_indptr", "segment_slots",
            "token_indices", "slice_offsets", "segment_count")
    missing = [k for k in keys if k not in routing]
    if missing or set(routing) - set(keys):
        raise TypeError(f"expected keyword arguments {keys}")
    _launch(entry, _native.fused_workspace_floats, x, a, b, output, *(routing[k] for k in keys),
            num_slices, numerics, workspace)


def base_gemm_workspace_floats(tokens: int, width: int, num_slices: int, capacity: int) -> int:
    """Elements of the FP32 workspace ``lora_base_gemm`` needs for these sizes."""
    return _native.lora_base_gemm_workspace_floats(tokens, width, num_slices, capacity)


@ExperimentalAPI(reason="Base projection GEMM with the LoRA delta in its mainloop; sm_100a tcgen05, FP32 numerics.")
def lora_base_gemm(
    x,
    weight,
    a,
    b,
    output,
    *,
    b_offsets,
    b_strides,
    ranks,
    scales,
    segment_indptr,
    segment_slots,
    token_indices,
    slice_offsets,
    segment_count,
    num_slices: int = 1,
    slice_widths=None,
    workspace=None,
) -> None:
    """``output = x @ weight.T + scale * B_g @ (A_g @ x[t])`` for every routed token, in one GEMM.

    The reference computes the base projection and then adds the LoRA delta into it
    (``lora_expand(..., base=)``, src/loraforge/ops/gemv.py:130-238), which reads and
    writes the output once more.  Here the delta is extra K steps of the base GEMM's
    accumulator, so ``output`` is written once and never read (its old contents are
    ignored).  ``weight`` is the base projection [N, width] (BF16, unit column stride);
    the LoRA operands and routing are those of ``lora_shrink_expand_prefill`` (route with
    ``group_tokens(..., chunk=128, runs=True)``).  Multi-slice outputs need every slice
    width to be a multiple of 256: pass ``slice_widths`` (host integers) or the offsets are
    read back once.  ``workspace``: FP32, ``base_gemm_workspace_floats(...)`` elements
    (allocated when omitted).
    """
    import torch

    _check_operands(x, a, b, output, b_offsets, b_strides, ranks, scales, segment_indptr, segment_slots,
                    token_indices, slice_offsets, segment_count, num_slices, "fp32")
    tensor_arg(weight, "weight", 2, torch.bfloat16, x.device)
    output_is_distinct(output, (weight,))
    if weight.stride(1) != 1 or weight.stride(0) % 8 or weight.shape[1] != x.shape[1] or weight.data_ptr() % 16:
        raise ValueError("weight must be [N, width] with unit column stride, 16-byte aligned rows")
    if weight.shape[0] != output.shape[1]:
        raise ValueError("weight rows must match the output width")
    if output.stride(0) % 8 or output.data_ptr() % 16:
        raise ValueError("output rows must be 16-byte aligned with a row stride multiple of 8")
    if num_slices > 1:
        widths = slice_widths
        if widths is None:
            bounds = slice_offsets.tolist()
            widths = [hi - lo for lo, hi in zip(bounds, bounds[1:])]
        if len(widths) != num_slices or any(w % 256 for w in widths[:-1]):
            raise ValueError("multi-slice lora_base_gemm needs slice widths that are multiples of 256")
    capacity = a.shape[1] // num_slices
    need = base_gemm_workspace_floats(x.shape[0], x.shape[1], num_slices, capacity)
    if workspace is None:
        workspace = torch.zeros(need, dtype=torch.float32, device=x.device)
    if (not isinstance(workspace, torch.Tensor) or workspace.dtype != torch.float32
            or workspace.device != x.device or workspace.numel() < need or workspace.data_ptr() % 16):
        raise ValueError(f"workspace must be a 16-byte aligned FP32 buffer of >= {need} elements on x's device")
    if x.shape[0] == 0:
        return
    with torch.cuda.device(x.device):
        _native.call(
            "lf_lora_base_gemm", x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), a.data_ptr(),
            b.data_ptr(), b_offsets.data_ptr(), b_strides.data_ptr(), output.data_ptr(), output.stride(0),
            segment_indptr.data_ptr(), segment_slots.data_ptr(), token_indices.data_ptr(), ranks.data_ptr(),
            scales.data_ptr(), slice_offsets.data_ptr(), segment_count.data_ptr(), workspace.data_ptr(),
            workspace.numel(), x.shape[0], x.shape[1], output.shape[1], num_slices, capacity, ranks.numel(),
            segment_slots.numel(), _native.stream_of(x.device),
        )
