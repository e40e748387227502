"""Padded-layout decode BGMV (SGLang's slot buffers) over the sm_100a C ABI.

Keeps the surface of ``loraforge.ops.gemv`` (src/loraforge/ops/gemv.py:46-238): call
signatures, the checks and their messages, FP32 / FP16 / BF16 activations.  Kernels:
``lf_bgmv_shrink`` groups the tokens of a slot into tiles of up to eight so each adapter's
A rows are read once per tile, accumulating in FP32; ``lf_bgmv_expand`` rounds the scaled
delta to the activation dtype before the base add.  Device values are never read on the
host, so warmed calls can be recorded into a CUDA graph.
"""

from __future__ import annotations

from loraforge_b200 import _native


def _inputs(x, weights, ranks, token_map):
    import torch

    if not all(isinstance(t, torch.Tensor) for t in (x, weights, ranks, token_map)):
        raise TypeError("inputs must be tensors")
    if x.ndim != 2 or weights.ndim != 3 or min(weights.shape) <= 0:
        raise ValueError("expected x[tokens, width] and nonempty weights[slots, rows, cols]")
    if x.device.type != "cuda" or any(t.device != x.device for t in (weights, ranks, token_map)):
        raise ValueError("all inputs must share a CUDA/ROCm device")
    if x.dtype not in (torch.float32, torch.float16, torch.bfloat16) or weights.dtype != x.dtype:
        raise ValueError("matching float32/float16/bfloat16 factors and activations required")
    if x.requires_grad or weights.requires_grad:
        raise ValueError("decode operators are inference-only")
    if not weights.is_contiguous() or x.stride(1) != 1:
        raise ValueError("weights must be contiguous and x must have unit column stride")
    if (
        ranks.ndim != 1
        or ranks.numel() != weights.shape[0]
        or token_map.ndim != 1
        or token_map.numel() < x.shape[0]
        or not ranks.is_contiguous()
        or not token_map.is_contiguous()
        or ranks.dtype not in (torch.int32, torch.int64)
        or token_map.dtype not in (torch.int32, torch.int64)
    ):
        raise ValueError("expected contiguous integer slot ranks and token mapping")


def _index_bits(t):
    import torch

    return 32 if t.dtype == torch.int32 else 64


def lora_shrink(x, weights, ranks, token_map, num_slices: int = 1):
    """Return z = A[token_map[t]] @ x[t] for every token, in x's dtype (a new tensor).

    ``weights`` holds each slot's A as [slices * capacity, width] rows; within a slot of
    rank r, slice s occupies rows s*r .. s*r + r - 1, and z's columns follow the same
    packing (the rest of each z row stays zero).  Sums are FP32, rounded once.  The
    device metadata is trusted, not read on the host: token_map values in [0, slots),
    ranks in [0, capacity]; a slot of rank 0 stands for the base model (zero row).
    """
    import torch

    _inputs(x, weights, ranks, token_map)
    if type(num_slices) is not int or num_slices <= 0 or weights.shape[1] % num_slices:
        raise ValueError("num_slices must divide the packed A row capacity")
    rank = weights.shape[1] // num_slices
    if not 1 <= rank <= 256 or x.shape[1] != weights.shape[2]:
        raise ValueError("rank capacity must be 1..256 and input widths must match")
    tokens, width = x.shape
    out = torch.zeros((tokens, num_slices * rank), device=x.device, dtype=x.dtype)
    if not tokens:
        return out
    if ranks.dtype != token_map.dtype:
        token_map = token_map.to(ranks.dtype)
    with torch.cuda.device(x.device):
        _native.call(
            "lf_bgmv_shrink",
            _native.dtype_code(x.dtype),
            x.data_ptr(),
            x.stride(0),
            weights.data_ptr(),
            out.data_ptr(),
            ranks.data_ptr(),
            token_map.data_ptr(),
            _index_bits(ranks),
            tokens,
            width,
            weights.shape[0],
            num_slices,
            rank,
            _native.stream_of(x.device),
        )
    return out


def lora_expand(x, weights, ranks, scales, token_map, offsets, max_slice_size: int, base=None):
    """Add scale * B[token_map[t]] @ z[t] into ``base`` (or a zero tensor) and return it.

    ``weights`` is B as [slots, total_output, capacity]; ``x`` is the packed z of
    ``lora_shrink``.  ``offsets`` (on the device) split the output columns into slices
    that start at zero, increase, and are at most ``max_slice_size`` wide; slice s reads
    z columns s*r .. s*r + r - 1.  The scaled delta is rounded to the activation dtype
    first and then added to the base, as in the reference operator.
    """
    import torch

    _inputs(x, weights, ranks, token_map)
    slots, width, rank = weights.shape
    if not x.is_contiguous() or not 1 <= rank <= 256:
        raise ValueError("intermediate must be contiguous; rank capacity must be 1..256")
    if (
        not isinstance(offsets, torch.Tensor)
        or offsets.device != x.device
        or offsets.ndim != 1
        or offsets.numel() < 2
        or not offsets.is_contiguous()
        or offsets.dtype not in (torch.int32, torch.int64)
    ):
        raise ValueError("expected contiguous integer device slice offsets")
    slices = offsets.numel() - 1
    if x.shape[1] != slices * rank:
        raise ValueError("intermediate width does not match slices and rank capacity")
    if (
        not isinstance(scales, torch.Tensor)
        or scales.device != x.device
        or scales.ndim != 1
        or scales.numel() != slots
        or not scales.is_contiguous()
        or scales.requires_grad
        or scales.dtype not in (torch.float32, torch.float16, torch.bfloat16)
    ):
        raise ValueError("expected contiguous floating device scales per slot")
    if type(max_slice_size) is not int or not 1 <= max_slice_size <= width:
        raise ValueError("max_slice_size must be within the output width")
    if base is not None and (
        not isinstance(base, torch.Tensor)
        or base.device != x.device
        or base.dtype != x.dtype
        or base.ndim != 2
        or base.shape[0] != x.shape[0]
        or base.shape[1] < width
        or base.requires_grad
        or base.stride(0) <= 0
        or base.stride(1) <= 0
    ):
        raise ValueError("base must match tokens, device and dtype with sufficient output width")
    if slices > 16:
        raise ValueError("at most 16 slices are supported")
    output = (
        torch.zeros((x.shape[0], width), device=x.device, dtype=x.dtype) if base is None else base
    )
    if not x.shape[0]:
        return output
    if ranks.dtype != token_map.dtype:
        token_map = token_map.to(ranks.dtype)
    with torch.cuda.device(x.device):
        _native.call(
            "lf_bgmv_expand",
            _native.dtype_code(x.dtype),
            x.data_ptr(),
            weights.data_ptr(),
            ranks.data_ptr(),
            scales.data_ptr(),
            _native.dtype_code(scales.dtype),
            token_map.data_ptr(),
            _index_bits(ranks),
            offsets.data_ptr(),
            _index_bits(offsets),
            output.data_ptr(),
            output.stride(0),
            output.stride(1),
            x.shape[0],
            width,
            slots,
            slices,
            rank,
            _native.stream_of(x.device),
        )
    return output
