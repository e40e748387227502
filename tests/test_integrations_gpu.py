"""The SGLang fleet backend on the B200 with real kernels: a stand-in for SGLang's chunked
backend carries batch_info tables built by the device grouping; the fused (gate/up) call is
checked against the FP32 oracle, the row-form (down) calls against the row operators'
two-rounding numerics."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from types import SimpleNamespace  # noqa: E402

from cases import values  # noqa: E402
from golden_io import bf16_bits, rel_l2  # noqa: E402
from oracle import cpu_reference as ref  # noqa: E402

from loraforge_b200.integrations import _sglang_fleet as fleet  # noqa: E402
from loraforge_b200.ops.grouping import group_tokens  # noqa: E402
from loraforge_b200.runtime.retained import RetainedLayout  # noqa: E402


class ChunkedBackend:
    def __init__(self, max_chunk_size=16):
        self.device = torch.device("cuda:0")
        self.max_chunk_size = max_chunk_size
        self.batch_info = None

    def prepare_lora_batch(self, forward_batch, weight_indices, lora_ranks, scalings, use_cuda_graph,
                           use_prefill_cuda_graph=False):
        self.batch_info = forward_batch.info


def native_unused(*args, **kwargs):
    raise AssertionError("no slot needs SGLang's kernels in this test")


def layer_ranks(name, r):
    parts = {"gate_up_proj": ("gate_proj", "up_proj"), "down_proj": ("down_proj",)}[name]
    return {f"base_model.model.model.layers.0.mlp.{p}.lora_A.weight": r for p in parts}


def padded_projection(slots, k, widths, cap, ranks, seed):
    """SGLang-style padded buffers filled per slot at the checkpoint rank (= cap)."""
    g = torch.Generator().manual_seed(seed)
    S, N = len(widths), sum(widths)
    a = torch.zeros(slots, S * cap, k, dtype=torch.bfloat16)
    b = torch.zeros(slots, N, cap, dtype=torch.bfloat16)
    for slot, r in enumerate(ranks):
        if r:
            for s in range(S):
                a[slot, s * cap : s * cap + r] = (torch.randn(r, k, generator=g) / k**0.5).bfloat16()
            b[slot, :, :r] = (torch.randn(N, r, generator=g) / r**0.5).bfloat16()
    return a.cuda(), b.cuda()


def batch(backend, slots_t, num_slots, chunk, decode):
    indptr, seg_slots, perm, count = group_tokens(slots_t, num_slots, chunk=chunk)
    nseg = int(count.item())
    info = SimpleNamespace(
        seg_indptr=indptr, weight_indices=seg_slots, permutation=perm, num_segments=nseg, use_cuda_graph=False,
        max_len=chunk, lora_ranks=None, scalings=(torch.rand(num_slots, generator=torch.Generator().manual_seed(5))
                                                 + 0.5).cuda(), req_weight_indices=slots_t,
    )
    mode = SimpleNamespace(is_decode=lambda: decode, is_extend=lambda: not decode)
    backend.prepare_lora_batch(SimpleNamespace(info=info, forward_mode=mode), None, None, None, False)
    return info


def expected_output(x, layout, slots_t, scales, base, widths, catalog_ranks):
    """FP32 oracle on the layout's repacked A and compact B (the slots' live factors)."""
    n = sum(widths)
    store = layout.store.float().cpu()
    boff, bucket = layout.boff.cpu().numpy(), layout.bucket.cpu().numpy()

    def rows(g):
        return store[boff[g] : boff[g] + n * bucket[g]].view(n, bucket[g])

    delta = ref.lora_delta_fp32(x.float().cpu().numpy(), layout.a.float().cpu(), rows, slots_t.cpu().numpy(),
                                np.asarray(catalog_ranks), scales.cpu().numpy(), np.cumsum((0, *widths)))
    return base.float().cpu().numpy() + delta


def row_numerics(x, layout, slots_t, scales, base, catalog_ranks):
    """The row operators' contract on one slice: z = bf16(A x), delta = bf16(scale * B z),
    out = bf16(y + delta) (src/loraforge/ops/csrc/lora_rows.cu:64,113)."""
    out = base.float().cpu().clone()
    n = base.shape[1]
    store = layout.store.float().cpu()
    boff, bucket = layout.boff.cpu().tolist(), layout.bucket.cpu().tolist()
    xf, a = x.float().cpu(), layout.a.float().cpu()
    for t, g in enumerate(slots_t.cpu().tolist()):
        r = catalog_ranks[g] if g >= 0 else 0
        if r == 0:
            continue
        z = (a[g, :r] @ xf[t]).bfloat16().float()
        b = store[boff[g] : boff[g] + n * bucket[g]].view(n, bucket[g])[:, :r]
        delta = (float(scales[g]) * (b @ z)).bfloat16().float()
        out[t] = (base[t].float().cpu() + delta).bfloat16().float()
    return out.bfloat16()


@pytest.mark.parametrize("decode,chunk,tokens", [(True, 16, 96), (False, 128, 700)])
def test_fleet_gate_up_and_down_through_b200_kernels(decode, chunk, tokens):
    slots_n, hidden, inter, cap = 6, 1024, 1536, 64
    ranks = [16, 64, 8, 32, 0, 4]
    rng = np.random.default_rng(int(decode))
    slots_t = torch.from_numpy(rng.integers(-1, slots_n, tokens).astype(np.int32)).cuda()
    catalog = {}
    gate_up = padded_projection(slots_n, hidden, (inter, inter), cap, ranks, 1)
    down = padded_projection(slots_n, inter, (hidden,), cap, ranks, 2)
    layouts = {}
    for name, (a, b) in (("gate_up_proj", gate_up), ("down_proj", down)):
        catalog = {f"ckpt{g}": layer_ranks(name, r) for g, r in enumerate(ranks)}
        layouts[name] = RetainedLayout(a, b, name, 0, catalog)
        for g, r in enumerate(ranks):
            layouts[name].load(f"ckpt{g}", g, cap)
    a_entries, b_entries = {}, {}
    backend_class = fleet.fleet_backend(ChunkedBackend, a_entries, b_entries, native_shrink=native_unused,
                                        native_expand=native_unused, policy=fleet.FleetPolicy())
    for layout in layouts.values():
        backend_class.bind_layout(layout)
    backend = backend_class(max_chunk_size=chunk)
    info = batch(backend, slots_t, slots_n, chunk, decode)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(tokens, hidden, generator=g).bfloat16().cuda()
    base = (torch.randn(tokens, 2 * inter, generator=g) * 0.5).bfloat16().cuda()
    e = layouts["gate_up_proj"]
    out = backend.run_gate_up_lora(x, e.a, e.b, None, base.clone(),
                                   output_offset_cpu=torch.tensor([0, inter, 2 * inter]))
    torch.cuda.synchronize()
    want = expected_output(x, e, slots_t, info.scalings, base, (inter, inter), ranks)
    gate = ref.fp32_gate(values(bf16_bits(out)), want)
    assert gate["excess"] <= 1e-2, gate
    # down_proj: separate A and B calls (row form, BF16 z like the reference's operators).
    h = torch.randn(tokens, inter, generator=g).bfloat16().cuda()
    base2 = (torch.randn(tokens, hidden, generator=g) * 0.5).bfloat16().cuda()
    d = layouts["down_proj"]
    z = backend.run_lora_a_sgemm(h, d.a, stack_num=1)
    out2 = backend.run_lora_b_sgemm(z, d.b, None, base2.clone(), output_offset_cpu=torch.tensor([0, hidden]))
    torch.cuda.synchronize()
    want2 = row_numerics(h, d, slots_t, info.scalings, base2, ranks)
    got2 = bf16_bits(out2)
    assert rel_l2(values(got2), values(bf16_bits(want2))) < 0.005  # the reference's row-operator gate
    assert np.mean(got2 == bf16_bits(want2)) > 0.95
    hits = backend.fleet_snapshot()["python_capture_eager_calls"]
    assert hits[f"fused_{'decode' if decode else 'prefill'}/gate_up_proj"] == 1
    assert hits["direct_shrink"] == 1 and hits[f"rowexpand_{'decode' if decode else 'prefill'}/down_proj"] == 1
