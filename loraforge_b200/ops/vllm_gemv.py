"""BGMV over vLLM's per-slice padded slot tensors, on the sm_100a C ABI.

Keeps the surface of ``loraforge.ops.vllm_gemv`` (src/loraforge/ops/vllm_gemv.py:49-159):
signatures, checks and messages; torch is imported only when a call is made.  The
reference's shrink splits K across programs that add with FP32 atomics, so its low bits
vary run to run; here every (token, rank row) sum runs in a fixed order (one warp per row,
or, for FP32 and unaligned operands, a K split over one thread-block cluster added in rank
order), and repeated calls give identical bits.  A route of -1 gives a zero intermediate
row and leaves the output row as it was.
"""

from loraforge_b200 import _native
from loraforge_b200.annotations import ExperimentalAPI


def _check(x, weights, routes):
    import torch

    if x.ndim != 2 or x.stride(-1) != 1 or x.device.type != "cuda":
        raise ValueError("expected GPU x[tokens, width] with contiguous columns")
    if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise ValueError("expected floating-point inputs")
    if (
        routes.device != x.device
        or routes.dtype != torch.int32
        or routes.shape != (x.shape[0],)
        or not routes.is_contiguous()
    ):
        raise ValueError("expected same-device contiguous int32 routes[tokens]")
    if not weights:
        raise ValueError("at least one weight slice is required")
    slots = weights[0].shape[0]
    for weight in weights:
        if (
            weight.ndim not in (3, 4)
            or (weight.ndim == 4 and weight.shape[1] != 1)
            or min(weight.shape) < 1
            or weight.shape[0] != slots
            or weight.stride(-1) != 1
            or weight.device != x.device
            or weight.dtype not in (torch.float32, torch.float16, torch.bfloat16)
        ):
            raise ValueError("invalid same-device padded weight slice")
    if any(t.requires_grad for t in (x, *weights)):
        raise ValueError("GEMV is inference-only")
    if len(weights) > 8:
        raise ValueError("at most 8 weight slices are supported")
    if any(w.dtype != x.dtype for w in weights):
        raise ValueError("weight slices must match the activation dtype")


def _descriptors(weights):
    table = (_native.SliceDesc * len(weights))()
    for i, w in enumerate(weights):
        table[i].ptr = w.data_ptr()
        table[i].slot_stride = w.stride(0)
        table[i].row_stride = w.stride(-2)
        table[i].rows = w.shape[-2]
    return table


@ExperimentalAPI(
    reason="Inference-only padded-slot GEMV; vLLM 0.26.0 layouts, FP32 intermediates, sm_100a CUDA."
)
def shrink(x, weights, out, routes, *, scale=1.0):
    """out[s, t] = scale * A_s[routes[t]] @ x[t] in FP32, for every weight slice s.

    Each slice's A is [slots, rank, width] or [slots, 1, rank, width]; ``out`` is
    [slices, tokens, rank] FP32.  Tokens routed to -1 get zero rows.
    """
    import torch

    _check(x, weights, routes)
    m, k = x.shape
    rank = weights[0].shape[-2]
    if k < 1 or not 1 <= rank <= 256:
        raise ValueError("width must be positive and rank must be in 1..256")
    if any(a.shape[-2:] != (rank, k) for a in weights):
        raise ValueError("A slice shape mismatch")
    if (
        out.device != x.device
        or out.dtype != torch.float32
        or out.shape != (len(weights), m, rank)
        or not out.is_contiguous()
        or out.requires_grad
    ):
        raise ValueError("expected contiguous same-device FP32 output buffer")
    with torch.cuda.device(x.device), torch.no_grad():
        out.zero_()
        if m == 0:
            return
        table = _descriptors(weights)
        _native.call(
            "lf_vllm_shrink",
            _native.dtype_code(x.dtype),
            x.data_ptr(),
            x.stride(0),
            table,
            len(weights),
            weights[0].shape[0],
            out.data_ptr(),
            routes.data_ptr(),
            m,
            k,
            rank,
            float(scale),
            _native.stream_of(x.device),
        )


@ExperimentalAPI(
    reason="Inference-only padded-slot GEMV; tolerance-based native parity, not full-model acceptance."
)
def expand(v, weights, y, routes, *, offset=0, add=True):
    """y[t, slice s columns] (+)= B_s[routes[t]] @ v[s, t], summed in FP32, cast once.

    Slice s writes the columns offset + (widths of the earlier slices) onward; with
    ``add`` the old y is added before the one cast.  Tokens routed to -1 and columns
    outside the slices keep their values, also with ``add=False``.
    """
    import torch

    _check(y, weights, routes)
    m = y.shape[0]
    rank = weights[0].shape[-1]
    if not 1 <= rank <= 256 or any(b.shape[-1] != rank for b in weights):
        raise ValueError("B slices must share rank in 1..256")
    if (
        v.device != y.device
        or v.dtype != torch.float32
        or v.shape != (len(weights), m, rank)
        or not v.is_contiguous()
        or v.requires_grad
    ):
        raise ValueError("expected same-device contiguous FP32 intermediate")
    if type(offset) is not int or offset < 0:
        raise ValueError("offset must be a nonnegative integer")
    if offset + sum(b.shape[-2] for b in weights) > y.shape[1]:
        raise ValueError("output slices exceed output width")
    with torch.cuda.device(y.device), torch.no_grad():
        if m == 0:
            return
        table = _descriptors(weights)
        _native.call(
            "lf_vllm_expand",
            _native.dtype_code(y.dtype),
            v.data_ptr(),
            table,
            len(weights),
            weights[0].shape[0],
            y.data_ptr(),
            y.stride(0),
            routes.data_ptr(),
            m,
            rank,
            offset,
            1 if add else 0,
            _native.stream_of(y.device),
        )
