"""Base projection with the LoRA delta in the same GEMM (lf_lora_base_gemm) on the B200.

``lora_base_gemm`` writes ``x @ W.T + scale * B_g @ (A_g @ x)`` in one tcgen05 GEMM.  The
reference is the FP32 product of the BF16 operands (W on the GPU in FP32 with TF32 off, the
LoRA delta from the CPU oracle's einsum over per-adapter gathers) and the gate is
BASELINE's: max|out - ref| beyond the BF16 rounding of the output <= 1e-2 RMS, and almost
every output equal to bf16(ref).  Cases: ragged sizes (a partial token tile and a partial
column tile, mixed ranks with TMA and padded cp.async B rows, tokens without adapter), two
slices, and BASELINE config 3's shapes (8192 tokens, 5120 x 5120, rank 64).
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

import bench  # noqa: E402
from oracle import cpu_reference as ref  # noqa: E402
from test_fused_gpu import fp32_reference  # noqa: E402
from test_prefill_gpu import geometric, prefill_case, routed  # noqa: E402

from loraforge_b200.ops.fused import lora_base_gemm  # noqa: E402


def base_fp32(x, w):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return (x.float() @ w.float().T).cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def check(out, expected, exact=0.99):
    gate = ref.fp32_gate(out.float().cpu().numpy(), expected)
    assert gate["excess"] <= 1e-2, gate
    assert gate["exact"] > exact, gate
    return gate


@pytest.mark.parametrize("widths,ranks", [((640,), [16, 32, 64, 7, 64, 32]), ((512, 512), [16] * 6)])
def test_ragged_sizes_against_fp32(widths, ranks):
    lengths = geometric(np.random.default_rng(4), 12, 80, total=1000)
    x, a, b, base, slots_t, meta, S = prefill_case(lengths, slots=len(ranks), k=1024, widths=widths,
                                                   ranks=ranks, seed=4, inactive=0.15)
    meta = routed(meta, slots_t, len(ranks), 128, runs=True)
    g = torch.Generator(device="cuda").manual_seed(5)
    w = (torch.randn(sum(widths), 1024, generator=g, device="cuda") / 32).bfloat16()
    out = torch.full_like(base, float("nan"))  # never read: old contents are ignored
    lora_base_gemm(x, w, a, b, out, **meta, num_slices=S, slice_widths=widths)
    torch.cuda.synchronize()
    zero = torch.zeros_like(base)
    expected = base_fp32(x, w) + fp32_reference(x, a, b, zero, slots_t, meta, S)
    check(out, expected)
    again = torch.zeros_like(base)
    lora_base_gemm(x, w, a, b, again, **meta, num_slices=S, slice_widths=widths)
    torch.cuda.synchronize()
    assert torch.equal(again, out)  # deterministic


def test_config3_shapes_against_fp32():
    host = bench.HostWorkload(3, 1234)
    wl = bench.Workload(host, torch.device("cuda", 0))
    p = wl.projections[0]
    from loraforge_b200.ops.grouping import group_tokens

    r = group_tokens(wl.slots, wl.nslots, chunk=128, runs=True)
    meta = dict(b_offsets=p.b_offsets, b_strides=p.b_strides, ranks=p.ranks, scales=p.scales,
                slice_offsets=p.slice_offsets, segment_indptr=r.segment_indptr,
                segment_slots=r.segment_slots, token_indices=r.token_indices, segment_count=r.segment_count)
    g = torch.Generator(device="cuda").manual_seed(6)
    w = (torch.randn(p.N, p.K, generator=g, device="cuda") / p.K**0.5).bfloat16()
    x = wl.x_of(p)
    out = torch.empty_like(p.y)
    lora_base_gemm(x, w, p.a, p.b, out, **meta, num_slices=p.S)
    torch.cuda.synchronize()
    expected = base_fp32(x, w) + bench.oracle_delta(host, p, host.x[p.host.K])
    check(out, expected)
