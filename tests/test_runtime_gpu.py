"""Adapter residency on the B200: GPUAdapterSlots' copy ordering, leases and slot reuse
(after tests/test_runtime_gpu.py:44-145 of the reference), and PEFT checkpoints served
end to end through the fused kernels from a ProjectionSlab and a RetainedLayout."""

import gc
import json

import numpy as np
import pytest

torch = pytest.importorskip("torch")
safetensors = pytest.importorskip("safetensors.torch")
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA device required"),
]

from cases import values  # noqa: E402
from golden_io import bf16_bits  # noqa: E402
from oracle import cpu_reference as ref  # noqa: E402

from loraforge_b200.ops.fused import lora_shrink_expand  # noqa: E402
from loraforge_b200.ops.grouping import group_tokens  # noqa: E402
from loraforge_b200.runtime import GPUAdapterSlots  # noqa: E402
from loraforge_b200.runtime.retained import RetainedLayout  # noqa: E402
from loraforge_b200.runtime.slab import ProjectionSlab, select_modules  # noqa: E402

ROUTING_KEYS = ("segment_indptr", "segment_slots", "token_indices", "segment_count")


def source(tmp_path, name, rank=3, dtype=torch.float32, rslora=False):
    directory = tmp_path / name
    directory.mkdir()
    (directory / "adapter_config.json").write_text(json.dumps(
        {"peft_type": "LORA", "r": rank, "lora_alpha": 6, "target_modules": ["proj"], "bias": "none",
         "use_rslora": rslora}))
    a = torch.arange(rank * 64).reshape(rank, 64).to(dtype) / 100
    b = torch.arange(32 * rank).reshape(32, rank).to(dtype) / 100
    safetensors.save_file({"base_model.model.proj.lora_A.weight": a, "base_model.model.proj.lora_B.weight": b},
                          directory / "adapter_model.safetensors")
    return directory, a, b


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rslora", [False, True])
def test_cross_stream_reload_and_lifetime(tmp_path, dtype, rslora):
    path, a, b = source(tmp_path, "first", dtype=dtype, rslora=rslora)
    other, _, _ = source(tmp_path, "other", rank=1, dtype=dtype)
    pool = GPUAdapterSlots(1, device="cuda:0")
    producer, consumer = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(producer):
        handle = pool.load(path, 0)
    with torch.cuda.stream(consumer):
        with pool.borrow(handle) as modules:
            (m,) = modules
            assert m.a.device == torch.device("cuda:0") and m.a.dtype == dtype
            assert m.rank == 3 and m.a.is_contiguous() and m.b.is_contiguous()
            result = (m.b.float() @ m.a.float()) * m.scaling
            with pytest.raises(RuntimeError, match="active"):
                pool.load(other, 0)
            with pytest.raises(RuntimeError, match="active"):
                pool.evict(handle)
        del modules, m
    with torch.cuda.stream(producer):
        replacement = pool.load(other, 0)
    with pytest.raises(ValueError, match="stale"):
        with pool.borrow(handle):
            pass
    pool.evict(replacement)
    del pool
    gc.collect()
    # Churn the allocator before waiting: the consumer's record keeps the block alive.
    churn = [torch.empty((3, 64), device="cuda:0", dtype=dtype) for _ in range(32)]
    consumer.synchronize()
    scale = 6 / (3**0.5 if rslora else 3)
    torch.testing.assert_close(result.cpu(), (b.float() @ a.float()) * scale)
    del churn


def test_failure_budget_and_exception_release(tmp_path):
    path, _, _ = source(tmp_path, "first", rank=1)
    large, _, _ = source(tmp_path, "large", rank=3)
    pool = GPUAdapterSlots(1, device="cuda:0", max_tensor_bytes=384)
    handle = pool.load(path, 0)
    assert pool.tensor_bytes == 384
    with pytest.raises(ValueError, match="limit"):
        pool.load(large, 0)
    with pytest.raises(ValueError, match="different"):
        with GPUAdapterSlots(1, device="cuda:0").borrow(handle):
            pass
    with pytest.raises(RuntimeError, match="consumer failure"):
        with pool.borrow(handle):
            raise RuntimeError("consumer failure")
    pool.collect()
    pool.evict(handle)
    assert pool.tensor_bytes == 0
    with pytest.raises(ValueError, match="stale"):
        pool.evict(handle)


def test_graph_capture_is_refused(tmp_path):
    path, _, _ = source(tmp_path, "first")
    pool = GPUAdapterSlots(1, device="cuda:0")
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        handle = pool.load(path, 0)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="graph capture"):
        with torch.cuda.graph(graph):
            pool.load(path, 0)
    with pool.borrow(handle):
        pass


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="two visible GPUs required")
@pytest.mark.parametrize("index", [0, 1])
def test_residency_device_guard(tmp_path, index):
    path, a, b = source(tmp_path, "adapter")
    previous = torch.cuda.current_device()
    other = 1 - index
    device = torch.device("cuda", index)
    try:
        torch.cuda.set_device(other)
        pool = GPUAdapterSlots(1, device=str(device))
        handle = pool.load(path, 0)
        assert torch.cuda.current_device() == other
        with torch.cuda.device(device), pool.borrow(handle) as modules:
            (module,) = modules
            assert module.a.device == module.b.device == device
            result = (module.b @ module.a) * module.scaling
        assert torch.cuda.current_device() == other
        pool.evict(handle)
        pool.collect()
        torch.testing.assert_close(result.cpu(), (b @ a) * 2)
    finally:
        torch.cuda.set_device(previous)


# ---------------------------------------------------------------- PEFT -> kernels

QKV = ("q_proj", "k_proj", "v_proj")


def qkv_checkpoint(root, name, seed, ranks, widths, k, alpha=16.0, rslora=False, dtype=torch.bfloat16):
    """A PEFT directory with q/k/v modules of layer 0 (per-module ranks via rank_pattern)."""
    g = torch.Generator().manual_seed(seed)
    directory = root / name
    directory.mkdir()
    tensors = {}
    for proj, r, w in zip(QKV, ranks, widths):
        key = f"base_model.model.model.layers.0.self_attn.{proj}"
        tensors[f"{key}.lora_A.weight"] = (torch.randn(r, k, generator=g) / k**0.5).to(dtype)
        tensors[f"{key}.lora_B.weight"] = (torch.randn(w, r, generator=g) / r**0.5).to(dtype)
    (directory / "adapter_config.json").write_text(json.dumps({
        "peft_type": "LORA", "r": ranks[0], "lora_alpha": alpha, "target_modules": list(QKV),
        "rank_pattern": {p: r for p, r in zip(QKV, ranks)}, "use_rslora": rslora}))
    safetensors.save_file(tensors, directory / "adapter_model.safetensors")
    return directory


def peft_reference(x, modules_by_slot, slots, base):
    """base + sum_s scaling_s * B_s @ (A_s @ x) per token, in FP32 from the PEFT factors."""
    xf = x.float().cpu()
    out = base.float().cpu().clone()
    for t, g in enumerate(slots.tolist()):
        if g < 0 or g not in modules_by_slot:
            continue
        col = 0
        for m in modules_by_slot[g]:
            w = m.b.shape[0]
            out[t, col : col + w] += m.scaling * (m.b.float().cpu() @ (m.a.float().cpu() @ xf[t]))
            col += w
    return out.numpy()


def test_peft_checkpoints_through_gpu_slots_and_slab(tmp_path):
    widths, k, slots_n, tokens = (1024, 256, 256), 1024, 6, 80
    specs = [((16, 16, 16), False), ((8, 4, 8), True), ((64, 64, 64), False), ((1, 2, 3), False),
             ((32, 32, 32), True), ((12, 12, 12), False)]
    pool = GPUAdapterSlots(slots_n, device="cuda:0")
    slab = ProjectionSlab(slots_n, k, widths, 64, device="cuda:0")
    loaded = {}
    for g, (ranks, rslora) in enumerate(specs):
        handle = pool.load(qkv_checkpoint(tmp_path, f"ad{g}", g, ranks, widths, k, rslora=rslora), g)
        with pool.borrow(handle) as modules:
            chosen = select_modules(modules, 0, QKV)
            slab.load(g, chosen)
            loaded[g] = [type(m)(m.name, m.a.cpu(), m.b.cpu(), m.alpha, m.use_rslora) for m in chosen]
    rng = np.random.default_rng(7)
    slots = torch.from_numpy(rng.integers(-1, slots_n, size=tokens).astype(np.int32)).cuda()
    x = torch.randn(tokens, k, generator=torch.Generator().manual_seed(3)).bfloat16().cuda()
    base = (torch.randn(tokens, sum(widths), generator=torch.Generator().manual_seed(4)) * 0.5).bfloat16().cuda()
    out = base.clone()
    ops = slab.operands()
    a = ops.pop("a")
    b = ops.pop("b")
    ops.update(zip(ROUTING_KEYS, group_tokens(slots, slots_n, chunk=16)))
    lora_shrink_expand(x, a, b, out, **ops)
    torch.cuda.synchronize()
    expected = peft_reference(x, loaded, slots.cpu(), base)
    gate = ref.fp32_gate(values(bf16_bits(out)), expected)
    assert gate["excess"] <= 1e-2, gate
    # An evicted adapter's slot cleared in the slab contributes nothing afterwards.
    slab.clear(2)
    out2 = base.clone()
    lora_shrink_expand(x, a, b, out2, **ops)
    torch.cuda.synchronize()
    inactive = (slots.cpu() == 2) | (slots.cpu() < 0)
    assert torch.equal(out2.cpu()[inactive], base.cpu()[inactive])


def test_retained_layout_feeds_fused_kernel():
    # SGLang-style padded buffers (capacity 64, slices of gate/up), three catalog
    # checkpoints of effective ranks 8, 24 and 100 (the last is left to native kernels).
    slots_n, k, width, cap, S = 4, 512, 768, 128, 2
    g = torch.Generator().manual_seed(9)
    a = torch.zeros(slots_n, S * cap, k, dtype=torch.bfloat16)
    b = torch.zeros(slots_n, S * width, cap, dtype=torch.bfloat16)

    def ranks(r):
        return {f"base_model.model.model.layers.0.mlp.{n}.lora_A.weight": r for n in ("gate_proj", "up_proj")}

    catalog = {"r8": ranks(8), "r24": ranks(24), "r100": ranks(100)}
    a, b = a.cuda(), b.cuda()
    e = RetainedLayout(a, b, "gate_up_proj", 0, catalog)
    factors = {}
    for slot, (path, r) in enumerate([("r8", 8), ("r24", 24), ("r100", 100)]):
        ckpt = 32 if r < 32 else cap  # the checkpoint's padded rank
        fa = (torch.randn(S, r, k, generator=g) / k**0.5).bfloat16()
        fb = (torch.randn(S * width, r, generator=g) / r**0.5).bfloat16()
        for s in range(S):  # native padded load: slice s at rows s*ckpt
            a[slot, s * ckpt : s * ckpt + r] = fa[s].cuda()
        b[slot, :, :r] = fb.cuda()
        e.load(path, slot, ckpt)
        factors[slot] = (fa, fb)
    x = torch.randn(64, k, generator=g).bfloat16().cuda()
    ids = torch.from_numpy(np.random.default_rng(2).integers(-1, slots_n, 64).astype(np.int32)).cuda()
    base = (torch.randn(64, S * width, generator=g) * 0.5).bfloat16().cuda()
    scales = torch.tensor([0.5, 2.0, 1.0, 1.0], dtype=torch.float32, device="cuda")
    meta = dict(e.kernel_operands(), scales=scales,
                slice_offsets=torch.tensor([0, width, 2 * width], dtype=torch.int32, device="cuda"))
    bstore = meta.pop("b")
    meta.update(zip(ROUTING_KEYS, group_tokens(ids, slots_n, chunk=16)))
    out = base.clone()
    lora_shrink_expand(x, e.a, bstore, out, **meta, num_slices=S)
    torch.cuda.synchronize()
    expected = base.float().cpu().clone()
    for t, slot in enumerate(ids.cpu().tolist()):
        if slot < 0 or slot not in factors or slot == 2:  # rank 100: not a B200-kernel slot
            continue
        fa, fb = factors[slot]
        for s in range(S):
            z = fa[s].float() @ x[t].float().cpu()
            expected[t, s * width : (s + 1) * width] += float(scales[slot]) * (fb[s * width : (s + 1) * width].float() @ z)
    gate = ref.fp32_gate(values(bf16_bits(out)), expected.numpy())
    assert gate["excess"] <= 1e-2, gate
    assert int(e.supported[2]) == 0 and int(e.unsupported[2]) == 100
