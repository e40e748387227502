"""Serving-framework registration and fleet dispatch on CPU, with stand-in modules for
SGLang and vLLM (after tests/test_sglang_registration.py, tests/test_vllm_registration.py
and the policy tests of tests/test_retained_layout.py in the reference).  The kernels
are replaced by recorders: these tests check which B200 entry point each call takes
and with which operands; the kernels' numerics are covered by the GPU suites."""

import subprocess
import sys
from types import ModuleType, SimpleNamespace

import pytest

torch = pytest.importorskip("torch")

from loraforge_b200.integrations import _sglang_fleet as fleet  # noqa: E402
from loraforge_b200.integrations import sglang  # noqa: E402
from loraforge_b200.integrations import vllm as vllm_integration  # noqa: E402
from loraforge_b200.runtime.retained import RetainedLayout  # noqa: E402

# ---------------------------------------------------------------- SGLang registration


def test_disabled_sglang_plugin_is_inert(monkeypatch):
    monkeypatch.delenv("LORAFORGE_SGLANG", raising=False)
    monkeypatch.setattr(sglang, "install_sglang_backend", lambda: pytest.fail("unexpected activation"))
    sglang.install()


def test_sglang_unsupported_version(monkeypatch):
    monkeypatch.setattr(sglang, "version", lambda name: "0.5.13")
    with pytest.raises(RuntimeError, match="0.5.22"):
        sglang.install_sglang_backend()


def _fake_registry(monkeypatch):
    path = "sglang.srt.lora.backend.lora_registry"
    for length in range(1, 6):
        name = ".".join(path.split(".")[:length])
        module = ModuleType(name)
        module.__path__ = []
        monkeypatch.setitem(sys.modules, name, module)
    registry = ModuleType(path)

    def native():
        pass

    native.__name__ = "create_triton_csgmv_backend"
    native.__module__ = path
    registry.LORA_SUPPORTED_BACKENDS = {"csgmv": native}
    monkeypatch.setitem(sys.modules, path, registry)
    return registry


def test_sglang_registration_idempotence_and_conflict(monkeypatch):
    registry = _fake_registry(monkeypatch)
    monkeypatch.setattr(sglang, "version", lambda name: "0.5.22")
    sglang.install_sglang_backend()
    assert registry.LORA_SUPPORTED_BACKENDS["csgmv"] is sglang.get_backend
    sglang.install_sglang_backend()
    registry.LORA_SUPPORTED_BACKENDS["csgmv"] = lambda: None
    with pytest.raises(RuntimeError, match="another plugin"):
        sglang.install_sglang_backend()


def test_sglang_enabled_entrypoint(monkeypatch):
    calls = []
    monkeypatch.setenv("LORAFORGE_SGLANG", "1")
    monkeypatch.setattr(sglang, "install_sglang_backend", lambda: calls.append(True))
    sglang.install()
    assert calls == [True]


@pytest.mark.parametrize("policy", ["compatible", "rank-aware", "fleet"])
def test_decode_policy_selection(monkeypatch, policy):
    monkeypatch.setenv("LORAFORGE_SGLANG_POLICY", policy)
    assert sglang._decode_policy() == policy


def test_unknown_decode_policy_rejected(monkeypatch):
    monkeypatch.setenv("LORAFORGE_SGLANG_POLICY", "unknown")
    with pytest.raises(ValueError, match="POLICY"):
        sglang._decode_policy()


# ---------------------------------------------------------------- vLLM registration


def test_disabled_vllm_plugin_is_dependency_free(monkeypatch):
    monkeypatch.delenv("LORAFORGE_VLLM", raising=False)
    code = """
import importlib.abc, sys
class Reject(importlib.abc.MetaPathFinder):
    def find_spec(self, fullname, path=None, target=None):
        if fullname.split('.')[0] in {'torch', 'triton', 'vllm'}:
            raise AssertionError(fullname)
sys.meta_path.insert(0, Reject())
from loraforge_b200.integrations.vllm import register
from loraforge_b200.ops.vllm_gemv import shrink, expand
register()
"""
    subprocess.run([sys.executable, "-c", code], check=True, cwd=str(_repo_root()))


def _repo_root():
    from pathlib import Path

    return Path(__file__).resolve().parents[1]


def test_vllm_alpha_metadata():
    from loraforge_b200.ops.vllm_gemv import expand, shrink

    for fn in (vllm_integration.install_vllm_backend, vllm_integration.register, shrink, expand):
        assert fn.__experimental_api__.stability == "alpha"


def test_vllm_unsupported_version(monkeypatch):
    monkeypatch.setattr(vllm_integration, "version", lambda _: "0.25.0")
    with pytest.raises(RuntimeError, match="exactly"):
        vllm_integration.install_vllm_backend()


@pytest.mark.parametrize("value", [0, -1, True, 1.5])
def test_vllm_invalid_threshold(value):
    with pytest.raises(ValueError, match="positive integer"):
        vllm_integration.install_vllm_backend(tokens_per_lora=value)


def test_vllm_opt_in(monkeypatch):
    calls = []
    monkeypatch.setenv("LORAFORGE_VLLM", "1")
    monkeypatch.setattr(vllm_integration, "install_vllm_backend", lambda: calls.append(1))
    vllm_integration.register()
    assert calls == [1]


def test_vllm_registration_conflicts(monkeypatch):
    name = "vllm.lora.punica_wrapper.punica_gpu"
    for length in range(1, 4):
        parent = ".".join(name.split(".")[:length])
        module = ModuleType(parent)
        module.__path__ = []
        monkeypatch.setitem(sys.modules, parent, module)
    module = ModuleType(name)

    class Wrapper:
        def add_lora_linear(self):
            pass

    Wrapper.add_lora_linear.__module__ = name
    module.PunicaWrapperGPU = Wrapper
    monkeypatch.setitem(sys.modules, name, module)
    monkeypatch.setattr(vllm_integration, "version", lambda _: "0.26.0")
    monkeypatch.setattr(vllm_integration, "_installed", None)
    monkeypatch.setattr(vllm_integration, "_operator", lambda: None)
    vllm_integration.install_vllm_backend()
    first = Wrapper.add_lora_linear
    vllm_integration.install_vllm_backend()
    assert Wrapper.add_lora_linear is first
    with pytest.raises(RuntimeError, match="conflict"):
        vllm_integration.install_vllm_backend(tokens_per_lora=8)
    Wrapper.add_lora_linear = lambda self: None
    with pytest.raises(RuntimeError, match="conflict"):
        vllm_integration.install_vllm_backend()
    monkeypatch.setattr(vllm_integration, "_installed", None)
    with pytest.raises(RuntimeError, match="foreign"):
        vllm_integration.install_vllm_backend()


def test_vllm_wrapper_routes_decode_and_defers_the_rest(monkeypatch):
    name = "vllm.lora.punica_wrapper.punica_gpu"
    module = ModuleType(name)
    native_calls, op_calls = [], []

    class Wrapper:
        def add_lora_linear(self, y, x, a, b, scale, slices, *, buffer=None, **kwargs):
            native_calls.append(kwargs)

    Wrapper.add_lora_linear.__module__ = name
    module.PunicaWrapperGPU = Wrapper
    monkeypatch.setitem(sys.modules, name, module)
    monkeypatch.setattr(vllm_integration, "version", lambda _: "0.26.0")
    monkeypatch.setattr(vllm_integration, "_installed", None)
    monkeypatch.setattr(vllm_integration, "_operator", lambda: lambda *args: op_calls.append(args))
    vllm_integration.install_vllm_backend(tokens_per_lora=2)
    wrapper = Wrapper()
    wrapper.lora_config = SimpleNamespace(specialize_active_lora=True)
    wrapper.token_mapping_meta = SimpleNamespace(meta_args=lambda n, flag: ("m",) * 7)
    a = [torch.zeros(4, 1, 8, 32)]
    b = [torch.zeros(4, 1, 64, 8)]
    x, y = torch.zeros(3, 32), torch.zeros(3, 64)
    wrapper.is_prefill = False
    wrapper.add_lora_linear(y, x, a, b, 0.5, (64,))
    assert len(op_calls) == 1 and op_calls[0][4] == 0.5 and op_calls[0][-1] == 2 and op_calls[0][-2] is True
    wrapper.is_prefill = True
    wrapper.add_lora_linear(y, x, a, b, 0.5, (64,), add_inputs=False)
    assert native_calls == [{"add_inputs": False}] and len(op_calls) == 1
    wrapper.is_prefill = False
    with pytest.raises(ValueError, match="widths"):
        wrapper.add_lora_linear(y, x, a, b, 0.5, (32,))


# ---------------------------------------------------------------- fleet policy and dispatch


def test_fleet_policy_rules():
    p = fleet.FleetPolicy()
    assert p.select("qkv_proj", "decode", 64, max_len=16, fused=True, slices=3) == dict(
        a="fused", b="fused", kernel="decode")
    assert p.select("gate_up_proj", "prefill", 4096, max_len=128, fused=True, slices=2)["kernel"] == "prefill"
    assert p.select("gate_up_proj", "prefill", 4096, max_len=256, fused=True, slices=2)["a"] == "direct"
    assert p.select("down_proj", "decode", 8, max_len=16)["b"] == "rowexpand"
    assert p.select("lm_head", "decode", 8)["a"] == "native"
    assert p.select("o_proj", "decode", 0)["b"] == "native"
    assert p.select("qkv_proj", "decode", 8, fused=True, slices=5)["a"] == "native"
    with pytest.raises(ValueError, match="numerics"):
        fleet.FleetPolicy(numerics="bf16")


def test_active_rank_classes_use_live_records():
    loaded = {0: {"rank": 0}, 1: {"rank": 3}, 2: {"rank": 128}}
    assert fleet.active_rank_classes(loaded, [0]) == (False, False)
    assert fleet.active_rank_classes(loaded, [0, 1]) == (True, False)
    assert fleet.active_rank_classes(loaded, [2]) == (False, True)
    assert fleet.active_rank_classes(loaded, [1, 3]) == (True, True)
    loaded[1] = {"rank": 64}
    assert fleet.active_rank_classes(loaded, [1]) == (True, False)
    loaded[1] = {"rank": 65}
    assert fleet.active_rank_classes(loaded, [1]) == (False, True)


@pytest.mark.parametrize("flag,enabled", [(None, False), ("0", False), ("1", True)])
def test_fleet_environment(tmp_path, monkeypatch, flag, enabled):
    import json

    manifest = tmp_path / "manifest.json"
    manifest.write_text(json.dumps({"adapters": [{"path": "adapter"}]}))
    monkeypatch.setenv("LORAFORGE_SGLANG_MANIFEST", str(manifest))
    monkeypatch.delenv("LORAFORGE_SGLANG_ACTIVE_PREFILL", raising=False)
    monkeypatch.delenv("LORAFORGE_SGLANG_NUMERICS", raising=False)
    if flag is not None:
        monkeypatch.setenv("LORAFORGE_SGLANG_ACTIVE_PREFILL", flag)
    monkeypatch.setattr(fleet, "read_rank_catalog", lambda paths: paths)
    monkeypatch.setattr(fleet, "create_backend", lambda catalog, **kwargs: (catalog, kwargs))
    assert fleet.backend_from_environment() == (["adapter"], {"active_prefill": enabled, "numerics": "fp32"})
    monkeypatch.setenv("LORAFORGE_SGLANG_ACTIVE_PREFILL", "yes")
    with pytest.raises(ValueError, match="must be 0 or 1"):
        fleet.backend_from_environment()
    monkeypatch.setenv("LORAFORGE_SGLANG_ACTIVE_PREFILL", "0")
    monkeypatch.setenv("LORAFORGE_SGLANG_NUMERICS", "bf16")
    with pytest.raises(ValueError, match="NUMERICS"):
        fleet.backend_from_environment()


class FakeChunkedBackend:
    """The parts of SGLang's ChunkedSgmvLoRABackend the fleet backend touches."""

    def __init__(self, max_chunk_size=16):
        self.device = torch.device("cpu")
        self.max_chunk_size = max_chunk_size
        self.batch_info = None

    def prepare_lora_batch(self, forward_batch, weight_indices, lora_ranks, scalings, use_cuda_graph,
                           use_prefill_cuda_graph=False):
        self.batch_info = forward_batch.info


def mlp_ranks(k):
    return {f"base_model.model.model.layers.0.mlp.{n}.lora_A.weight": k for n in ("gate_proj", "up_proj")}


@pytest.fixture
def fleet_setup(monkeypatch):
    """A fleet backend over CPU stand-ins, with every kernel call recorded."""
    import loraforge_b200.ops.fused as fused_ops
    import loraforge_b200.ops.grouping as grouping_ops
    import loraforge_b200.ops.rowexpand as rowexpand_ops

    calls = []

    def recorder(name, result_index=None):
        def record(*args, **kwargs):
            calls.append((name, args, kwargs))
            return None if result_index is None else args[result_index]
        return record

    monkeypatch.setattr(fused_ops, "lora_shrink_expand", recorder("fused_decode"))
    monkeypatch.setattr(fused_ops, "lora_shrink_expand_prefill", recorder("fused_prefill"))
    monkeypatch.setattr(rowexpand_ops, "direct_shrink", recorder("direct_shrink", 2))
    monkeypatch.setattr(rowexpand_ops, "row_expand", recorder("row_expand", 4))
    monkeypatch.setattr(grouping_ops, "segment_routes",
                        lambda indptr, slots, perm, count, n: torch.full((n,), 7, dtype=torch.int32))
    monkeypatch.setattr(grouping_ops, "group_tokens",
                        lambda routes, slots, chunk: ("ip16", "slots16", torch.zeros(routes.numel()), "count16"))
    monkeypatch.setattr(fleet, "require_sm100", lambda device: None)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)

    def native_shrink(x, weights, info, slices):
        calls.append(("native_shrink", info.lora_ranks))
        return torch.zeros(x.shape[0], weights.shape[1], dtype=x.dtype)

    def native_expand(z, weights, info, offsets, max_slice, output, slice_offsets_cpu=None):
        calls.append(("native_expand", info.lora_ranks))
        return output if output is not None else torch.zeros(z.shape[0], weights.shape[1], dtype=z.dtype)

    a_entries, b_entries = {}, {}
    backend_class = fleet.fleet_backend(FakeChunkedBackend, a_entries, b_entries, native_shrink=native_shrink,
                                        native_expand=native_expand, policy=fleet.FleetPolicy())
    a = torch.zeros(3, 2 * 128, 64, dtype=torch.bfloat16)
    b = torch.zeros(3, 2 * 96, 128, dtype=torch.bfloat16)
    layout = RetainedLayout(a, b, "gate_up_proj", 0, {"small": mlp_ranks(16), "huge": mlp_ranks(100)})
    layout.load("small", 1, 16)
    backend_class.bind_layout(layout)
    return backend_class, layout, calls


def make_batch(backend, tokens, max_len, decode=True):
    info = SimpleNamespace(
        seg_indptr=torch.zeros(tokens + 1, dtype=torch.int32), weight_indices=torch.zeros(tokens, dtype=torch.int32),
        permutation=torch.arange(tokens, dtype=torch.int32), num_segments=2, use_cuda_graph=False,
        max_len=max_len, lora_ranks=torch.tensor([0, 16, 100], dtype=torch.int32),
        scalings=torch.ones(3), req_weight_indices=torch.zeros(tokens, dtype=torch.int32),
    )
    mode = SimpleNamespace(is_decode=lambda: decode, is_extend=lambda: not decode)
    backend.prepare_lora_batch(SimpleNamespace(info=info, forward_mode=mode), [0, 1], None, None, False)
    return info


def test_fleet_fused_decode_and_prefill_calls(fleet_setup):
    backend_class, layout, calls = fleet_setup
    backend = backend_class()
    info = make_batch(backend, 8, 16)
    assert backend._fleet_segments.tolist() == [2]
    x = torch.zeros(8, 64, dtype=torch.bfloat16)
    base = torch.zeros(8, 192, dtype=torch.bfloat16)
    cpu = torch.tensor([0, 96, 192])
    out = backend.run_gate_up_lora(x, layout.a, layout.b, "offsets", base, output_offset_cpu=cpu)
    assert out is base
    # Slot 2's rank-100 checkpoint is in the catalog, so the native kernels run for it first
    # with every other slot masked out, then one fused call serves the rest.
    names = [c[0] for c in calls]
    assert names == ["native_shrink", "native_expand", "fused_decode"]
    assert calls[0][1] is layout.unsupported
    _, args, kwargs = calls[2]
    assert args[1] is layout.a and args[2] is layout.store and args[3] is base
    assert kwargs["ranks"] is layout.supported and kwargs["b_strides"] is layout.bucket
    assert kwargs["segment_indptr"] is info.seg_indptr and kwargs["token_indices"] is info.permutation
    assert kwargs["workspace"] == "builtin" and kwargs["num_slices"] == 2
    assert kwargs["slice_offsets"].tolist() == [0, 96, 192]
    calls.clear()
    make_batch(backend, 512, 128, decode=False)
    backend.run_gate_up_lora(torch.zeros(512, 64, dtype=torch.bfloat16), layout.a, layout.b, "offsets",
                             torch.zeros(512, 192, dtype=torch.bfloat16), output_offset_cpu=cpu)
    assert [c[0] for c in calls] == ["native_shrink", "native_expand", "fused_prefill"]
    assert backend.fleet_snapshot()["python_capture_eager_calls"]["fused_prefill/gate_up_proj"] == 1


def test_fleet_row_form_and_unknown_buffers(fleet_setup):
    backend_class, layout, calls = fleet_setup
    backend = backend_class()
    make_batch(backend, 40, 32, decode=False)
    x = torch.zeros(40, 64, dtype=torch.bfloat16)
    z = backend.run_lora_a_sgemm(x, layout.a, stack_num=2)
    assert [c[0] for c in calls] == ["native_shrink", "direct_shrink"]
    _, args, _ = calls[1]
    assert args[3].tolist() == [7] * 40 and args[4] is layout.supported and args[6] == 64
    calls.clear()
    cpu = torch.tensor([0, 96, 192])
    backend.run_lora_b_sgemm(z, layout.b, "offsets", torch.zeros(40, 192, dtype=torch.bfloat16),
                             output_offset_cpu=cpu)
    assert [c[0] for c in calls] == ["native_expand", "row_expand"]
    _, args, _ = calls[1]
    # SGLang's 32-token chunks are re-grouped on the device into 16-token segments.
    assert args[5] == "ip16" and args[6] == "slots16" and args[11] == "count16" and args[12] == 128
    calls.clear()
    other = torch.zeros(3, 256, 64, dtype=torch.bfloat16)  # a buffer with no layout
    backend.run_lora_a_sgemm(x, other, stack_num=2)
    assert [c[0] for c in calls] == ["native_shrink"]


def test_fleet_backend_guards(fleet_setup, monkeypatch):
    backend_class, layout, calls = fleet_setup
    with pytest.raises(ValueError, match="max_lora_chunk_size"):
        backend_class(max_chunk_size=256)
    monkeypatch.setattr(fleet, "require_sm100", lambda device: (_ for _ in ()).throw(ValueError("sm_100")))
    with pytest.raises(ValueError, match="sm_100"):
        backend_class()


def test_pool_hooks_build_and_load_layouts(tmp_path):
    class Pool:
        tp_size, enable_lora_overlap_loading = 1, False

        def init_buffers(self):
            self.A_buffer = {"gate_up_proj": [torch.zeros(2, 2 * 32, 16, dtype=torch.bfloat16), None]}
            self.B_buffer = {"gate_up_proj": [torch.zeros(2, 2 * 24, 32, dtype=torch.bfloat16), None]}

        def load_lora_weight_to_buffer(self, uid, buffer_id, adapter):
            self.last = (uid, buffer_id)

    path = str((tmp_path / "ckpt").resolve())
    a_entries, b_entries = {}, {}
    fleet.install_pool_hooks(Pool, {path: mlp_ranks(8)}, a_entries, b_entries)
    with pytest.raises(RuntimeError, match="another backend"):
        fleet.install_pool_hooks(Pool, {}, {}, {})
    pool = Pool()
    pool.init_buffers()
    (layout,) = pool._loraforge_layouts
    assert a_entries[pool.A_buffer["gate_up_proj"][0].data_ptr()] is layout
    adapter = SimpleNamespace(config=SimpleNamespace(path=path, r=32))
    pool.load_lora_weight_to_buffer("u1", 1, adapter)
    assert pool.last == ("u1", 1) and layout.supported.tolist() == [0, 8]
    with pytest.raises(ValueError, match="catalog"):
        pool.load_lora_weight_to_buffer("u2", 0, SimpleNamespace(config=SimpleNamespace(path="/elsewhere", r=8)))
    assert pool.last == ("u1", 1)  # refused before SGLang's own load
    pool.load_lora_weight_to_buffer(None, 1, None)
    assert layout.supported.tolist() == [0, 0]
    bad = Pool()
    bad.tp_size = 2
    with pytest.raises(ValueError, match="TP=1"):
        bad.init_buffers()
