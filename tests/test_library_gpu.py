"""The torch.library ops on the B200: same bits as the direct calls, eager, under
torch.compile (the op is an opaque node: fullgraph compiles without a break) and in a
captured CUDA graph."""

import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from cases import row_case  # noqa: E402
from test_fused_gpu import decode_case  # noqa: E402

from loraforge_b200.ops import row_expand, row_shrink  # noqa: E402
from loraforge_b200.ops.fused import lora_shrink_expand, workspace_floats  # noqa: E402
from loraforge_b200.ops.library import register  # noqa: E402

KEYS = ("b_offsets", "b_strides", "ranks", "scales", "segment_indptr", "segment_slots",
        "token_indices", "slice_offsets", "segment_count")


def test_row_ops_match_direct_calls():
    ops = register()
    x, a, z, b, storage, output, routes, meta = row_case(slices=2, width=512)
    z1, z2 = z.clone(), z.clone()
    row_shrink(x, a, z1, routes, meta["ranks"], num_slices=2)
    ops.row_shrink(x, a, z2, routes, meta["ranks"], 2, 64)
    torch.cuda.synchronize()
    assert torch.equal(z1, z2)
    y1 = torch.zeros(x.shape[0], output.shape[1], dtype=torch.bfloat16, device="cuda")
    y2 = y1.clone()
    row_expand(z1, b, y1, **meta)
    torch.ops.loraforge_b200.row_expand(z1, b, y2, *(meta[k] for k in KEYS), None, 256)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


def test_fused_op_under_compile_and_graph():
    ops = register()
    x, a, b, base, slots_t, meta, S, cap = decode_case(seed=31)
    ws = torch.zeros(workspace_floats(x.shape[0], x.shape[1], S, cap), device="cuda")
    want = base.clone()
    lora_shrink_expand(x, a, b, want, **meta, num_slices=S)

    def step(x, a, b, y, ws):
        ops.lora_shrink_expand(x, a, b, y, *(meta[k] for k in KEYS), S, "fp32", ws)
        return y

    compiled = torch.compile(step, fullgraph=True)
    got = base.clone()
    compiled(x, a, b, got, ws)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    out = base.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step(x, a, b, out, ws)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(x, a, b, out, ws)
    out.copy_(base)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
