"""The allocation-free fused entry point (lf_fused_shrink_expand_noalloc) on the B200.

Some callers cannot allocate device memory (an engine that has handed all free GPU
memory to its own cache pool, or a cgo/JNI/FFI host without the framework's
allocator).  For them the library offers a variant of the fused shrink/expand whose
scratch is a fixed buffer compiled into the library.  This file is named so that it
is collected last: the variant must give the same output as the workspace entry
point, on two calls in a row (the buffer keeps the previous call's contents), both
in a fresh process and after every other test has run.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from loraforge_b200 import _native  # noqa: E402
from loraforge_b200.ops.fused import lora_shrink_expand  # noqa: E402
from loraforge_b200.ops.grouping import group_tokens  # noqa: E402


def make_case(seed, tokens=96, slots=24, k=4096, widths=(4096, 1024, 1024), rank=16):
    g = torch.Generator().manual_seed(seed)
    S, N = len(widths), sum(widths)
    x = torch.randn(tokens, k, generator=g).bfloat16().cuda()
    a = (torch.randn(slots, S * rank, k, generator=g) / k**0.5).bfloat16().cuda()
    b = (torch.randn(slots * N * rank, generator=g) / rank**0.5).bfloat16().cuda()
    ids = torch.randint(-1, slots, (tokens,), generator=g, dtype=torch.int32).cuda()
    base = (torch.randn(tokens, N, generator=g) * 0.5).bfloat16().cuda()
    meta = dict(
        b_offsets=torch.arange(slots, dtype=torch.int64).cuda() * (N * rank),
        b_strides=torch.full((slots,), rank, dtype=torch.int32).cuda(),
        ranks=torch.full((slots,), rank, dtype=torch.int32).cuda(),
        scales=(torch.rand(slots, generator=g) + 0.5).cuda(),
        slice_offsets=torch.tensor(np.cumsum((0, *widths)), dtype=torch.int32).cuda(),
    )
    routing = group_tokens(ids, slots, chunk=16)
    meta.update(
        segment_indptr=routing.segment_indptr,
        segment_slots=routing.segment_slots,
        token_indices=routing.token_indices,
        segment_count=routing.segment_count,
    )
    return x, a, b, base, meta, S, rank


def call_noalloc(x, a, b, out, meta, S, rank, numerics=0):
    _native.call(
        "lf_fused_shrink_expand_noalloc",
        x.data_ptr(), x.stride(0), a.data_ptr(), b.data_ptr(),
        meta["b_offsets"].data_ptr(), meta["b_strides"].data_ptr(),
        out.data_ptr(), out.stride(0),
        meta["segment_indptr"].data_ptr(), meta["segment_slots"].data_ptr(),
        meta["token_indices"].data_ptr(), meta["ranks"].data_ptr(),
        meta["scales"].data_ptr(), meta["slice_offsets"].data_ptr(),
        meta["segment_count"].data_ptr(),
        x.shape[0], x.shape[1], out.shape[1], S, rank, meta["ranks"].numel(),
        meta["segment_slots"].numel(), numerics, _native.stream_of(x.device),
    )


@pytest.mark.parametrize("numerics", ["fp32", "reference"])
def test_matches_workspace_entry_point_on_consecutive_calls(numerics):
    code = {"fp32": 0, "reference": 1}[numerics]
    # Different problems back to back (other slice counts, widths and token counts):
    # every call starts from the previous call's leftovers in the shared buffers.
    cases = (
        (1, 96, 4096, (4096, 1024, 1024)),
        (2, 96, 4096, (14336, 14336)),
        (3, 40, 14336, (4096,)),
        (4, 160, 4096, (4096, 1024, 1024)),
    )
    for seed, tokens, k, widths in cases:
        x, a, b, base, meta, S, rank = make_case(seed, tokens=tokens, k=k, widths=widths)
        expected = base.clone()
        lora_shrink_expand(x, a, b, expected, **meta, num_slices=S, numerics=numerics)
        got = base.clone()
        call_noalloc(x, a, b, got, meta, S, rank, code)
        torch.cuda.synchronize()
        torch.testing.assert_close(got, expected, rtol=0, atol=0)
    assert _native.device_wait_timeouts(reset=True) == 0


def test_rejects_sizes_beyond_the_built_in_buffer():
    x, a, b, base, meta, S, rank = make_case(3, tokens=8)
    big_tokens = 1 << 20  # needs far more than 4 Mi floats of scratch
    with pytest.raises(RuntimeError, match="built-in"):
        _native.call(
            "lf_fused_shrink_expand_noalloc",
            x.data_ptr(), x.stride(0), a.data_ptr(), b.data_ptr(),
            meta["b_offsets"].data_ptr(), meta["b_strides"].data_ptr(),
            base.data_ptr(), base.stride(0),
            meta["segment_indptr"].data_ptr(), meta["segment_slots"].data_ptr(),
            meta["token_indices"].data_ptr(), meta["ranks"].data_ptr(),
            meta["scales"].data_ptr(), meta["slice_offsets"].data_ptr(),
            meta["segment_count"].data_ptr(),
            big_tokens, x.shape[1], base.shape[1], S, rank, meta["ranks"].numel(),
            meta["segment_slots"].numel(), 0, _native.stream_of(x.device),
        )


def test_builtin_workspace_keyword_on_two_sizes_in_a_row():
    # Calls of different batch sizes one after another share the built-in scratch.
    cases = [make_case(seed, tokens=tokens) for seed, tokens in ((5, 64), (6, 200))]
    for _ in range(2):
        for x, a, b, base, meta, S, rank in cases:
            want = base.clone()
            lora_shrink_expand(x, a, b, want, **meta, num_slices=S)
            out = base.clone()
            lora_shrink_expand(x, a, b, out, **meta, num_slices=S, workspace="builtin")
            torch.cuda.synchronize()
            torch.testing.assert_close(out, want, rtol=0, atol=0)
    x, a, b, base, meta, S, rank = cases[0]
    with pytest.raises(ValueError, match="builtin"):
        lora_shrink_expand(x, a, b, base.clone(), **meta, num_slices=S, workspace="static")
    assert _native.device_wait_timeouts(reset=True) == 0
