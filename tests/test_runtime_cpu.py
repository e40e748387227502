"""Adapter residency on CPU: the PEFT loader's refusals, the CPU slot pool, handle
rules, and RetainedLayout against the reference's own outputs for the known-answer
sequence of tests/test_retained_layout.py:24-61 (tests/golden/retained_layout.npz)."""

import json
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
safetensors = pytest.importorskip("safetensors.torch")

from golden_io import bf16_bits, load, to_torch  # noqa: E402

from loraforge_b200.adapters import load_peft_adapter, write_manifest  # noqa: E402
from loraforge_b200.runtime import AdapterSlots, GPUAdapterSlots, SlotHandle  # noqa: E402
from loraforge_b200.runtime.gpu import pack_layout  # noqa: E402
from loraforge_b200.runtime.retained import (  # noqa: E402
    RetainedLayout,
    bucket_of,
    effective_rank,
    read_rank_catalog,
)


def write_adapter(root, name, *, rank=3, rslora=False, config=None, tensors=None, dtype=torch.float32):
    directory = root / name
    directory.mkdir()
    cfg = {"peft_type": "LORA", "r": rank, "lora_alpha": 6, "target_modules": ["proj"],
           "bias": "none", "use_rslora": rslora}
    cfg.update(config or {})
    (directory / "adapter_config.json").write_text(json.dumps(cfg))
    if tensors is None:
        tensors = {
            "base_model.model.proj.lora_A.weight": torch.arange(rank * 5).float().reshape(rank, 5).to(dtype),
            "base_model.model.proj.lora_B.weight": torch.ones(4, rank, dtype=dtype),
        }
    safetensors.save_file(tensors, directory / "adapter_model.safetensors")
    return directory


# ---------------------------------------------------------------- PEFT loader


@pytest.mark.parametrize("rslora", [False, True])
def test_loader_scaling_and_patterns(tmp_path, rslora):
    tensors = {
        "base_model.model.layers.0.proj.lora_A.weight": torch.randn(8, 6),
        "base_model.model.layers.0.proj.lora_B.weight": torch.randn(5, 8),
        "base_model.model.block.proj.lora_A.weight": torch.randn(2, 6),
        "base_model.model.block.proj.lora_B.weight": torch.randn(5, 2),
    }
    path = write_adapter(tmp_path, "a", rank=8, rslora=rslora, tensors=tensors,
                         config={"rank_pattern": {"block.proj": 2}, "alpha_pattern": {"block.proj": 7}})
    adapter = load_peft_adapter(path)
    got = {m.name: (m.rank, m.alpha, m.scaling) for m in adapter.modules}
    root = math.sqrt if rslora else (lambda r: r)
    assert got == {"block.proj": (2, 7.0, 7 / root(2)), "layers.0.proj": (8, 6.0, 6 / root(8))}
    assert [m.name for m in adapter.modules] == sorted(got)


@pytest.mark.parametrize(
    "change, message",
    [
        ({"peft_type": "IA3"}, "only PEFT LORA"),
        ({"use_dora": True}, "use_dora"),
        ({"bias": "all"}, "bias"),
        ({"surprise": 1}, "unsupported configuration fields"),
        ({"modules_to_save": ["head"]}, "modules_to_save"),
        ({"init_lora_weights": "pissa"}, "initialization"),
        ({"lora_dropout": 2}, "dropout"),
        ({"lora_alpha": float("inf")}, "finite"),
        ({"target_modules": []}, "target_modules"),
        ({"target_modules": ["other"]}, "target/exclude"),
        ({"exclude_modules": ["proj"]}, "target/exclude"),
        ({"rank_pattern": {"proj": 0}}, "rank_pattern"),
        ({"r": 4}, "configured rank"),
        ({"runtime_config": {"ephemeral_gpu_offload": True}}, "runtime_config"),
    ],
)
def test_loader_refusals(tmp_path, change, message):
    with pytest.raises(ValueError, match=message):
        load_peft_adapter(write_adapter(tmp_path, "bad", config=change))


def test_loader_tensor_refusals(tmp_path):
    ok_a = torch.ones(3, 5)
    cases = {
        "key": ({"model.proj.lora_A.weight": ok_a}, "unsupported tensor key"),
        "pair": ({"base_model.model.proj.lora_A.weight": ok_a}, "incomplete A/B pair"),
        "nan": ({"base_model.model.proj.lora_A.weight": ok_a * float("nan"),
                 "base_model.model.proj.lora_B.weight": torch.ones(4, 3)}, "nonfinite"),
        "dtype": ({"base_model.model.proj.lora_A.weight": ok_a.double(),
                   "base_model.model.proj.lora_B.weight": torch.ones(4, 3).double()}, "layout or dtype"),
    }
    for name, (tensors, message) in cases.items():
        with pytest.raises(ValueError, match=message):
            load_peft_adapter(write_adapter(tmp_path, name, tensors=tensors))
    with pytest.raises(FileNotFoundError):
        load_peft_adapter(tmp_path / "missing")


def test_manifest_integrity(tmp_path):
    path = write_adapter(tmp_path, "m")
    write_manifest(path)
    assert load_peft_adapter(path).modules[0].rank == 3
    (path / "adapter_model.safetensors").write_bytes(b"corrupt")
    with pytest.raises(ValueError, match="integrity"):
        load_peft_adapter(path)


# ---------------------------------------------------------------- CPU slot pool


@pytest.mark.parametrize("rslora", [False, True])
def test_reuse_scaling_and_ownership(tmp_path, rslora):
    first = write_adapter(tmp_path, "first", rslora=rslora)
    second = write_adapter(tmp_path, "second", rank=1)
    pool = AdapterSlots(1)
    handle = pool.load(first, 0)
    (module,) = pool.resolve(handle)
    assert module.rank == 3 and module.a.is_contiguous() and module.b.is_contiguous()
    assert module.scaling == pytest.approx(6 / (3**0.5 if rslora else 3))
    assert pool.tensor_bytes == (3 * 5 + 4 * 3) * 4
    module.a.zero_()
    assert pool.resolve(handle)[0].a.sum() > 0
    replacement = pool.load(second, 0)
    for call in (pool.resolve, pool.evict):
        with pytest.raises(ValueError, match="stale"):
            call(handle)
    assert pool.resolve(replacement)[0].rank == 1
    pool.evict(replacement)
    assert pool.tensor_bytes == 0


def test_failed_load_preserves_occupant_and_budget(tmp_path):
    small = write_adapter(tmp_path, "small", rank=1)
    large = write_adapter(tmp_path, "large", rank=3)
    pool = AdapterSlots(2, max_tensor_bytes=36)
    handle = pool.load(small, 0)
    for path, slot in [(large, 0), (small, 1), (tmp_path / "missing", 0)]:
        with pytest.raises((ValueError, FileNotFoundError)):
            pool.load(path, slot)
        assert pool.resolve(handle)[0].rank == 1 and pool.tensor_bytes == 36
    with pytest.raises(ValueError, match="different pool"):
        AdapterSlots(2).resolve(handle)
    with pytest.raises(ValueError, match="different pool"):
        pool.resolve(SlotHandle("elsewhere", 0, 1))
    pool.evict(handle)
    assert pool.load(small, 1).slot == 1


def test_concurrent_independent_slots(tmp_path):
    from concurrent.futures import ThreadPoolExecutor

    path = write_adapter(tmp_path, "shared")
    pool = AdapterSlots(4)
    with ThreadPoolExecutor(max_workers=4) as pool_threads:
        handles = list(pool_threads.map(lambda i: pool.load(path, i), range(4)))
    assert pool.tensor_bytes == 4 * 108 and len({h.generation for h in handles}) == 1
    with ThreadPoolExecutor(max_workers=4) as pool_threads:
        list(pool_threads.map(pool.evict, handles))
    assert pool.tensor_bytes == 0


@pytest.mark.parametrize("capacity", [0, -1, True, 1.5])
def test_capacity(capacity):
    with pytest.raises(ValueError, match="capacity"):
        AdapterSlots(capacity)


@pytest.mark.parametrize("slot", [-1, 1, True, 0.5])
def test_invalid_slot(tmp_path, slot):
    with pytest.raises(ValueError, match="slot"):
        AdapterSlots(1).load(tmp_path / "absent", slot)


@pytest.mark.parametrize("limit", [-1, True, 0.5])
def test_invalid_limit(limit):
    with pytest.raises(ValueError, match="max_tensor_bytes"):
        AdapterSlots(1, max_tensor_bytes=limit)


@pytest.mark.parametrize("device", ["cpu", "cuda", "meta"])
def test_gpu_pool_requires_indexed_device(device):
    with pytest.raises(ValueError, match="explicitly"):
        GPUAdapterSlots(1, device=device)


def test_gpu_pack_layout_is_one_aligned_block(tmp_path):
    adapter = load_peft_adapter(write_adapter(tmp_path, "p", rank=3, dtype=torch.bfloat16))
    spans, total = pack_layout(adapter.modules)
    assert spans == [(0, 3 * 5 * 2), (256, 4 * 3 * 2)] and total == 512


# ---------------------------------------------------------------- RetainedLayout


def mlp_ranks(k, other=None, layer=0):
    return {
        f"base_model.model.model.layers.{layer}.mlp.{name}.lora_A.weight": value
        for name, value in (("gate_proj", k), ("up_proj", k if other is None else other))
    }


def test_retained_layout_matches_reference_outputs():
    g = load("retained_layout.npz")
    a, b = to_torch(g["a0"]), to_torch(g["b"])
    original_a = a.clone()
    catalog = {"low": mlp_ranks(3, 2), "high": mlp_ranks(32), "fallback": mlp_ranks(128)}
    e = RetainedLayout(a, b, "gate_up_proj", 0, catalog)
    assert np.array([e.regions[k] for k in ("low", "high", "fallback")]).tolist() == g["regions"].tolist()
    assert e.max_rank == int(g["max_rank"]) and e.store.numel() == int(g["store_numel"])
    assert e.has_high and e.has_unsupported
    pointers = [t.data_ptr() for t in (e.a, e.b, e.store, e.rank, e.low, e.high, e.boff, e.bucket)]
    for i, (path, slot, rank) in enumerate([("low", 1, 128), ("fallback", 1, 128), ("high", 1, 128), (None, 1, 0)]):
        a[1].copy_(original_a[1])
        e.load(path, slot, rank)
        assert np.array_equal(bf16_bits(a), g[f"step{i}_a"]), i
        assert np.array_equal(bf16_bits(e.store), g[f"step{i}_store"]), i
        for field in ("rank", "supported", "unsupported", "low", "high", "bucket", "boff"):
            assert np.array_equal(getattr(e, field).numpy(), g[f"step{i}_{field}"]), (i, field)
    assert pointers == [t.data_ptr() for t in (e.a, e.b, e.store, e.rank, e.low, e.high, e.boff, e.bucket)]
    assert np.array_equal(bf16_bits(b), g["b"])
    before = a.clone()
    with pytest.raises(ValueError, match="catalog"):
        e.load("unknown", 1, 128)
    with pytest.raises(ValueError, match="does not fit"):
        e.load("high", 1, 16)
    with pytest.raises(ValueError, match="slot out of range"):
        e.load("high", 2, 128)
    assert torch.equal(a, before)
    effective = [effective_rank(mlp_ranks(3, 7), "gate_up_proj", 0),
                 effective_rank(mlp_ranks(3), "gate_up_proj", 1),
                 effective_rank(mlp_ranks(3), "qkv_proj", 0)]
    assert effective == g["effective_rank"].tolist()


def test_retained_layout_kernel_operands_and_errors():
    a = torch.zeros(3, 2 * 64, 16, dtype=torch.bfloat16)
    b = torch.zeros(3, 24, 64, dtype=torch.bfloat16)
    e = RetainedLayout(a, b, "gate_up_proj", 0, {"x": mlp_ranks(12), "y": mlp_ranks(64)})
    assert e.regions == {"x": (0, 16, 12), "y": (24 * 16, 64, 64)}
    e.load("x", 2, 64)
    ops = e.kernel_operands()
    assert ops["b"] is e.store and ops["ranks"] is e.supported
    assert ops["b_offsets"].tolist() == [0, 0, 0] and ops["b_strides"].tolist() == [0, 0, 16]
    assert e.kernel_operands(rank_class="low")["ranks"].tolist() == [0, 0, 12]
    with pytest.raises(ValueError, match="rank_class"):
        e.kernel_operands(rank_class="high")
    with pytest.raises(ValueError, match="BF16 3D"):
        RetainedLayout(a.float(), b, "gate_up_proj", 0, {})
    with pytest.raises(ValueError, match="capacity"):
        RetainedLayout(a[:, :100], b, "gate_up_proj", 0, {})
    with pytest.raises(ValueError, match="exceeds native capacity"):
        RetainedLayout(a, b, "gate_up_proj", 0, {"z": mlp_ranks(65)})
    assert [bucket_of(k) for k in (0, 1, 2, 3, 5, 16, 17, 64)] == [1, 1, 2, 4, 8, 16, 32, 64]


def test_read_rank_catalog(tmp_path):
    key = "base_model.model.model.layers.0.mlp.gate_proj.lora_{}.weight"
    a = torch.zeros(8, 16)
    a[:3] = 1
    b = torch.zeros(32, 8)
    b[:, :3] = 1
    path = tmp_path / "ckpt"
    path.mkdir()
    (path / "adapter_config.json").write_text(json.dumps({"r": 8, "lora_alpha": 8}))
    safetensors.save_file({key.format("A"): a, key.format("B"): b}, path / "adapter_model.safetensors")
    assert read_rank_catalog([path]) == {str(path.resolve()): {key.format("A"): 8}}
    (path / "compression.json").write_text(json.dumps({"module_ranks": {key.format("A"): 3}}))
    catalog = read_rank_catalog([path])
    assert catalog[str(path.resolve())][key.format("A")] == 3
    assert effective_rank(catalog[str(path.resolve())], "gate_up_proj", 0) == 3
    (path / "compression.json").write_text(json.dumps({"module_ranks": {key.format("A"): 2}}))
    with pytest.raises(ValueError, match="truncates nonzero"):
        read_rank_catalog([path])
    (path / "adapter_config.json").write_text(json.dumps({"r": 8, "lora_alpha": 8, "use_rslora": True}))
    with pytest.raises(ValueError, match="SGLang padding"):
        read_rank_catalog([path])
    with pytest.raises(ValueError, match="nonempty"):
        read_rank_catalog([])


# ---------------------------------------------------------------- ProjectionSlab


def qkv_modules(seed, ranks, widths=(32, 8, 8), k=24, alphas=(8, 8, 8), rslora=False):
    from loraforge_b200.adapters import AdapterModule

    g = torch.Generator().manual_seed(seed)
    names = ("q_proj", "k_proj", "v_proj")
    return [
        None if r == 0 else AdapterModule(
            f"model.layers.3.self_attn.{n}", torch.randn(r, k, generator=g).bfloat16(),
            torch.randn(w, r, generator=g).bfloat16(), float(al), rslora,
        )
        for n, r, w, al in zip(names, ranks, widths, alphas)
    ]


def slab_delta_weight(slab, slot):
    """scale * B_s @ A_s of every slice, read back from the slab's packed tensors."""
    k, bucket = int(slab.ranks[slot]), int(slab.b_strides[slot])
    start = int(slab.b_offsets[slot])
    b = slab.b[start : start + slab.out_width * bucket].view(slab.out_width, bucket).float()
    parts, row0 = [], 0
    for s, w in enumerate(slab.slice_widths):
        a = slab.a[slot, s * k : (s + 1) * k].float()
        parts.append(float(slab.scales[slot]) * b[row0 : row0 + w, :k] @ a)
        row0 += w
    return parts


def test_projection_slab_packs_heterogeneous_slices():
    from loraforge_b200.runtime.slab import ProjectionSlab, select_modules

    slab = ProjectionSlab(4, 24, (32, 8, 8), 16, device="cpu")
    assert slab.region % 8 == 0 and slab.b_offsets.tolist() == [0, 768, 1536, 2304]
    cases = {1: qkv_modules(1, (6, 3, 0), alphas=(12, 3, 1)), 3: qkv_modules(2, (16, 16, 16), rslora=True)}
    for slot, modules in cases.items():
        slab.load(slot, modules)
    assert slab.ranks.tolist() == [0, 6, 0, 16] and slab.b_strides.tolist() == [0, 8, 0, 16]
    for slot, modules in cases.items():
        for part, m in zip(slab_delta_weight(slab, slot), modules):
            want = torch.zeros_like(part) if m is None else m.scaling * m.b.float() @ m.a.float()
            torch.testing.assert_close(part, want, rtol=1e-2, atol=1e-2)
    # Slab rows beyond the slot's rank stay zero, so a lower-rank reload leaves no residue.
    slab.load(3, qkv_modules(3, (2, 2, 2)))
    assert not slab.a[3, 6:].any() and int(slab.ranks[3]) == 2
    slab.clear(1)
    assert slab.ranks.tolist() == [0, 0, 0, 2] and 1 not in slab.loaded
    modules = qkv_modules(4, (4, 4, 4))
    assert select_modules(modules, 3, ("k_proj", "o_proj")) == [modules[1], None]
    with pytest.raises(ValueError, match="capacity"):
        slab.load(0, qkv_modules(5, (32, 1, 1)))
    with pytest.raises(ValueError, match="shape"):
        slab.load(0, qkv_modules(6, (4, 4, 4), widths=(8, 8, 8)))
    with pytest.raises(ValueError, match="slot"):
        slab.load(4, modules)
