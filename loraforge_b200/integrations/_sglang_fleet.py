"""Retained-rank SGLang fleet backend on B200 kernels (drop-in for the reference's
``_sglang_fleet``, src/loraforge/integrations/_sglang_fleet.py:1-523).

Same plumbing as the reference: a frozen catalog of checkpoint ranks
(``LORAFORGE_SGLANG_MANIFEST``), pool hooks on SGLang's ``LoRAMemoryPool`` that
build one ``RetainedLayout`` per (projection, layer) over SGLang's padded A/B
buffers and keep it loaded, and a ``ChunkedSgmvLoRABackend`` subclass whose four
methods dispatch per call.  What runs is B200-first:

* ``run_qkv_lora`` / ``run_gate_up_lora`` make ONE fused call per projection
  (shrink -> FP32 z -> expand; ``lora_shrink_expand`` on the library's built-in
  workspace for segments of <= 16 tokens, ``lora_shrink_expand_prefill`` on the
  tcgen05 tiles for <= 128), reading SGLang's segment table as-is;
* ``run_lora_a_sgemm`` / ``run_lora_b_sgemm`` (o_proj, down_proj, ...) run the row
  form: ``direct_shrink`` on per-token routes recovered on the device from the
  segment table, then ``row_expand`` over segments of <= 16 tokens (re-grouped on the
  device when SGLang's chunks are longer);
* slots whose retained rank exceeds 64 keep SGLang's native kernels (with the
  other slots' ranks masked to zero), as in the reference.

The reference's MI250X guard becomes an sm_100 guard, and its tuned dispatch table
becomes ``FleetPolicy``'s shape rules; no routing value is read on the host.
"""

from __future__ import annotations

import copy
import json
import os
import weakref
from collections import Counter
from pathlib import Path

from loraforge_b200.runtime.retained import MAX_KERNEL_RANK, RetainedLayout, read_rank_catalog

PROJECTIONS = ("qkv_proj", "gate_up_proj", "o_proj", "down_proj", "in_proj_qkvz", "in_proj_ba", "out_proj")
DECODE_MAX_LEN = 16
PREFILL_MAX_LEN = 128


class FleetPolicy:
    """Kernel choice for one LoRA call on the B200.

    ``select`` returns ``a`` / ``b`` (``"fused"``, ``"direct"`` / ``"rowexpand"``, or
    ``"native"``) and ``kernel`` (``"decode"`` or ``"prefill"`` for fused calls):

    * projections outside ``PROJECTIONS``, empty batches and slices beyond four stay
      native;
    * a fused call (QKV or gate/up) whose segments hold at most 16 tokens uses the
      decode kernels, at most 128 the prefill tcgen05 kernels; longer chunks fall
      back to the row form;
    * every other call uses the row form.
    ``numerics`` is passed to the fused kernels (``"fp32"`` keeps z in FP32).
    """

    def __init__(self, *, numerics: str = "fp32"):
        if numerics not in ("fp32", "reference"):
            raise ValueError("numerics must be 'fp32' or 'reference'")
        self.numerics = numerics

    def select(self, name, phase, tokens, *, max_len=None, fused=False, slices=1):
        native = dict(a="native", b="native", kernel=None)
        if name not in PROJECTIONS or tokens < 1 or not 1 <= slices <= 4 or phase not in ("decode", "prefill"):
            return native
        longest = max_len or DECODE_MAX_LEN
        if fused and longest <= DECODE_MAX_LEN:
            return dict(a="fused", b="fused", kernel="decode")
        if fused and longest <= PREFILL_MAX_LEN:
            return dict(a="fused", b="fused", kernel="prefill")
        return dict(a="direct", b="rowexpand", kernel=None)


def _masked(info, ranks):
    result = copy.copy(info)
    result.lora_ranks = ranks
    return result


def active_rank_classes(loaded, slots):
    """(kernel ranks, native ranks) present among ``slots`` from the CPU slot records.

    A slot without a record counts as both.  Device ranks are never read here (that
    would synchronise every projection).
    """
    kernel = native = False
    for slot in slots:
        entry = loaded.get(slot)
        if entry is None:
            return True, True
        kernel |= 0 < entry["rank"] <= MAX_KERNEL_RANK
        native |= entry["rank"] > MAX_KERNEL_RANK
        if kernel and native:
            break
    return kernel, native


def _fused_output_ok(output, dtype) -> bool:
    # The fused kernels write 8-byte groups of output columns.
    return (
        output.dtype == dtype
        and output.stride(1) == 1
        and output.stride(0) % 4 == 0
        and output.data_ptr() % 8 == 0
    )


def require_sm100(device) -> None:
    """The fleet kernels are built for sm_100a only."""
    import torch

    if torch.version.hip or torch.cuda.get_device_capability(device) != (10, 0):
        raise ValueError("the LoRAForge B200 fleet backend requires an sm_100 (B200) GPU")


def install_pool_hooks(pool_class, catalog, a_entries, b_entries):
    """Wrap SGLang's pool so every (projection, layer) gets a loaded RetainedLayout."""
    if getattr(pool_class, "_loraforge_fleet", False):
        raise RuntimeError("Fleet pool hooks already belong to another backend instance")
    old_init, old_load = pool_class.init_buffers, pool_class.load_lora_weight_to_buffer

    def init_pool(self, *args, **kwargs):
        if self.tp_size != 1 or self.enable_lora_overlap_loading:
            raise ValueError("Fleet requires TP=1 and non-overlapping adapter loading")
        old_init(self, *args, **kwargs)
        self._loraforge_layouts = []
        for name, per_layer in self.A_buffer.items():
            if name not in PROJECTIONS:
                raise ValueError(f"unsupported Fleet projection: {name}")
            for layer, (a, b) in enumerate(zip(per_layer, self.B_buffer[name], strict=True)):
                if a is None or b is None:
                    continue
                entry = RetainedLayout(a, b, name, layer, catalog)
                self._loraforge_layouts.append(entry)
                a_entries[a.data_ptr()] = entry
                b_entries[b.data_ptr()] = entry
        from loraforge_b200.ops.rowexpand import rowexpand_extension

        rowexpand_extension()  # load the library before any graph capture

    def load_pool(self, uid, buffer_id, adapter, *args, **kwargs):
        path = None if uid is None else str(Path(adapter.config.path).resolve())
        rank = 0 if uid is None else int(adapter.config.r)
        for e in self._loraforge_layouts:  # refuse before SGLang overwrites its buffers
            e.validate_load(path, rank)
        result = old_load(self, uid, buffer_id, adapter, *args, **kwargs)
        for e in self._loraforge_layouts:
            e.load(path, buffer_id, rank)
        return result

    pool_class.init_buffers = init_pool
    pool_class.load_lora_weight_to_buffer = load_pool
    pool_class._loraforge_fleet = True


def create_backend(catalog, *, active_prefill=False, numerics="fp32"):
    """Install the pool hooks and return the fleet backend class (SGLang 0.5.22 names)."""
    from sglang.kernels.ops.lora.dense.chunked_sgmv_expand import chunked_sgmv_lora_expand_forward
    from sglang.kernels.ops.lora.dense.chunked_sgmv_shrink import chunked_sgmv_lora_shrink_forward
    from sglang.srt.lora.backend.chunked_backend import ChunkedSgmvLoRABackend
    from sglang.srt.lora.mem_pool import LoRAMemoryPool

    a_entries, b_entries = weakref.WeakValueDictionary(), weakref.WeakValueDictionary()
    install_pool_hooks(LoRAMemoryPool, catalog, a_entries, b_entries)
    return fleet_backend(
        ChunkedSgmvLoRABackend, a_entries, b_entries,
        native_shrink=chunked_sgmv_lora_shrink_forward, native_expand=chunked_sgmv_lora_expand_forward,
        policy=FleetPolicy(numerics=numerics), active_prefill=active_prefill,
    )


def fleet_backend(base, a_entries, b_entries, *, native_shrink, native_expand, policy, active_prefill=False):
    """The backend class over ``base``; the SGLang kernels are injected for the native ranks."""
    import torch

    from loraforge_b200.ops.fused import lora_shrink_expand, lora_shrink_expand_prefill
    from loraforge_b200.ops.grouping import group_tokens, segment_routes
    from loraforge_b200.ops.rowexpand import direct_shrink, row_expand

    def expand_native(z, weights, info, offsets, max_slice, output, cpu):
        return native_expand(z, weights, info, offsets, max_slice, output, slice_offsets_cpu=cpu)

    class FleetBackend(base):
        supports_prefill_cuda_graph = False  # prefill workspaces are allocated per call

        def __init__(self, *args, **kwargs):
            super().__init__(*args, **kwargs)
            require_sm100(self.device)
            if self.max_chunk_size > PREFILL_MAX_LEN:
                raise ValueError(f"Fleet requires max_lora_chunk_size <= {PREFILL_MAX_LEN}")
            self._fleet_segments = torch.zeros(1, dtype=torch.int32, device=self.device)
            self._fleet_decode = False
            self._fleet_hits = Counter()
            self._fleet_active_prefill = active_prefill
            self._fleet_prefill_slots = None
            self._fleet_routes = None
            self._fleet_rows16 = None

        def prepare_lora_batch(self, forward_batch, weight_indices, lora_ranks, scalings, use_cuda_graph,
                               use_prefill_cuda_graph=False):
            # Invalidate first, including graph preparation and failed prepares.
            self._fleet_prefill_slots = self._fleet_routes = self._fleet_rows16 = None
            super().prepare_lora_batch(forward_batch, weight_indices, lora_ranks, scalings, use_cuda_graph,
                                       use_prefill_cuda_graph)
            info = self.batch_info
            self._fleet_segments.fill_(info.weight_indices.shape[0] if info.use_cuda_graph else info.num_segments)
            self._fleet_decode = forward_batch.forward_mode.is_decode()
            if (
                self._fleet_active_prefill
                and forward_batch.forward_mode.is_extend()
                and not use_cuda_graph
                and not use_prefill_cuda_graph
                and not torch.cuda.is_current_stream_capturing()
                and isinstance(weight_indices, (list, tuple))
                and all(type(slot) is int for slot in weight_indices)
            ):
                self._fleet_prefill_slots = tuple(dict.fromkeys(weight_indices))

        # ---------------------------------------------------------------- helpers
        def _phase(self):
            return "decode" if self._fleet_decode else "prefill"

        def _routes(self, tokens):
            if self._fleet_routes is None or self._fleet_routes.numel() != tokens:
                info = self.batch_info
                self._fleet_routes = segment_routes(info.seg_indptr, info.weight_indices, info.permutation,
                                                    self._fleet_segments, tokens)
            return self._fleet_routes

        def _rows16(self, tokens, slots):
            # Segments of <= 16 tokens for the row expand; SGLang's own when short enough.
            info = self.batch_info
            if (info.max_len or DECODE_MAX_LEN) <= DECODE_MAX_LEN:
                return info.seg_indptr, info.weight_indices, info.permutation, self._fleet_segments
            if self._fleet_rows16 is None or self._fleet_rows16[2].numel() != tokens:
                self._fleet_rows16 = tuple(group_tokens(self._routes(tokens), slots, chunk=DECODE_MAX_LEN))
            return self._fleet_rows16

        def _needs(self, e):
            # (kernel slots active, native slots active) for this batch.
            need_kernel, need_native = True, e.has_unsupported
            if self._fleet_prefill_slots is not None and not torch.cuda.is_current_stream_capturing():
                need_kernel, active_native = active_rank_classes(e.loaded, self._fleet_prefill_slots)
                need_native = need_native and active_native
            return need_kernel, need_native

        def _slice_offsets(self, e, cpu, device):
            if not hasattr(e, "slice_offsets"):
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError("warm each projection before capturing Fleet graphs")
                e.slice_offsets = torch.tensor(cpu.tolist(), device=device, dtype=torch.int32)
            return e.slice_offsets

        # ---------------------------------------------------------------- fused calls
        def _fused(self, x, wa, wb, offsets, max_slice, base_output, slices, cpu, native_call):
            e = a_entries.get(wa.data_ptr())
            info = self.batch_info
            cfg = policy.select(e.name if e is not None else None, self._phase(), x.shape[0],
                                max_len=info.max_len, fused=True, slices=slices)
            eligible = (
                e is not None
                and b_entries.get(wb.data_ptr()) is e
                and cfg["a"] == "fused"
                and cpu is not None
                and x.dtype == torch.bfloat16
                and (base_output is None or _fused_output_ok(base_output, x.dtype))
            )
            if not eligible:
                self._fleet_hits["native_fused_call"] += 1
                return native_call(info)
            need_kernel, need_native = self._needs(e)
            if base_output is None:
                base_output = torch.zeros((x.shape[0], wb.shape[1]), dtype=x.dtype, device=x.device)
            if need_native:
                base_output = native_call(_masked(info, e.unsupported), base_output)
            if not need_kernel:
                return base_output
            kwargs = dict(
                **e.kernel_operands(), scales=info.scalings, segment_indptr=info.seg_indptr,
                segment_slots=info.weight_indices, token_indices=info.permutation,
                slice_offsets=self._slice_offsets(e, cpu, x.device), segment_count=self._fleet_segments,
                num_slices=slices, numerics=policy.numerics,
            )
            b = kwargs.pop("b")
            if x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
                x = x.clone(memory_format=torch.contiguous_format)  # fresh, 16-byte aligned rows
            self._fleet_hits[f"fused_{cfg['kernel']}/{e.name}"] += 1
            if cfg["kernel"] == "decode":
                lora_shrink_expand(x, e.a, b, base_output, **kwargs, workspace="builtin")
            else:
                lora_shrink_expand_prefill(x, e.a, b, base_output, **kwargs)
            return base_output

        def run_qkv_lora(self, x, qkv_lora_a, qkv_lora_b, output_offset, max_qkv_out_dim, base_output=None,
                         n_slices=3, *args, **kwargs):
            cpu = kwargs.get("output_offset_cpu")

            def native(info, output=None):
                z = native_shrink(x, qkv_lora_a, info, n_slices)
                return expand_native(z, qkv_lora_b, info, output_offset, max_qkv_out_dim,
                                     base_output if output is None else output, cpu)

            return self._fused(x, qkv_lora_a, qkv_lora_b, output_offset, max_qkv_out_dim, base_output, n_slices,
                               cpu, native)

        def run_gate_up_lora(self, x, gate_up_lora_a, gate_up_lora_b, output_offset, base_output=None, *args,
                             **kwargs):
            cpu = kwargs.get("output_offset_cpu")
            max_slice = gate_up_lora_b.shape[-2] // 2

            def native(info, output=None):
                z = native_shrink(x, gate_up_lora_a, info, 2)
                return expand_native(z, gate_up_lora_b, info, output_offset, max_slice,
                                     base_output if output is None else output, cpu)

            return self._fused(x, gate_up_lora_a, gate_up_lora_b, output_offset, max_slice, base_output, 2,
                               cpu, native)

        # ---------------------------------------------------------------- row form
        def run_lora_a_sgemm(self, x, weights, pruned_batch_info=None, stack_num=1, *args, **kwargs):
            info = self.batch_info if pruned_batch_info is None else pruned_batch_info
            e = a_entries.get(weights.data_ptr())
            cfg = policy.select(e.name if e is not None else None, self._phase(), x.shape[0],
                                max_len=info.max_len, slices=stack_num)
            eligible = (
                e is not None
                and cfg["a"] == "direct"
                and info is self.batch_info
                and x.dtype == torch.bfloat16
                and x.shape[1] % 8 == 0
            )
            if not eligible:
                self._fleet_hits["native_shrink"] += 1
                return native_shrink(x, weights, info if e is None else _masked(info, e.rank), stack_num)
            x = x.contiguous()
            z = (
                native_shrink(x, weights, _masked(info, e.unsupported), stack_num)
                if e.has_unsupported
                else torch.empty((x.shape[0], weights.shape[1]), dtype=x.dtype, device=x.device)
            )
            self._fleet_hits["direct_shrink"] += 1
            return direct_shrink(x, weights, z, self._routes(x.shape[0]), e.supported, stack_num,
                                 min(e.max_rank, e.capacity))

        def run_lora_b_sgemm(self, x, weights, output_offset, base_output=None, pruned_batch_info=None, *args,
                             **kwargs):
            info = self.batch_info if pruned_batch_info is None else pruned_batch_info
            cpu = kwargs.get("output_offset_cpu")
            e = b_entries.get(weights.data_ptr())
            slices = None if cpu is None else cpu.numel() - 1
            cfg = policy.select(e.name if e is not None else None, self._phase(), x.shape[0],
                                max_len=info.max_len, slices=slices or 0)
            eligible = (
                e is not None
                and cfg["b"] == "rowexpand"
                and info is self.batch_info
                and x.dtype == torch.bfloat16
                and x.is_contiguous()
                and (base_output is None or (base_output.dtype == x.dtype and base_output.stride(1) == 1))
            )
            if not eligible:
                self._fleet_hits["native_expand"] += 1
                masked = info if e is None else _masked(info, e.rank)
                return expand_native(x, weights, masked, output_offset, weights.shape[-2], base_output, cpu)
            if base_output is None:
                base_output = torch.zeros((x.shape[0], weights.shape[1]), dtype=x.dtype, device=x.device)
            need_kernel, need_native = self._needs(e)
            if need_native:
                base_output = expand_native(x, weights, _masked(info, e.unsupported), output_offset,
                                            weights.shape[-2], base_output, cpu)
            if not need_kernel:
                return base_output
            indptr, seg_slots, perm, count = self._rows16(x.shape[0], e.b.shape[0])
            self._fleet_hits[f"rowexpand_{self._phase()}/{e.name}"] += 1
            return row_expand(x, e.store, e.boff, e.bucket, base_output, indptr, seg_slots, perm, e.supported,
                              info.scalings, self._slice_offsets(e, cpu, x.device), count, e.capacity)

        def fleet_snapshot(self):
            entries = list(a_entries.values())
            return dict(
                policy="fleet",
                numerics=policy.numerics,
                active_prefill=self._fleet_active_prefill,
                python_capture_eager_calls=dict(self._fleet_hits),
                modules=len(entries),
                shadow_bytes=sum(e.store.numel() * e.store.element_size() for e in entries),
                loaded={f"{e.layer}:{e.name}": e.loaded for e in entries},
            )

    # Test hook: bind a layout without SGLang's pool (framework-free lifecycle checks).
    FleetBackend.bind_layout = staticmethod(
        lambda e: (a_entries.__setitem__(e.a.data_ptr(), e), b_entries.__setitem__(e.b.data_ptr(), e))
    )
    return FleetBackend


def backend_from_environment():
    """Build the backend from ``LORAFORGE_SGLANG_MANIFEST`` and the opt-in switches."""
    active_prefill = os.environ.get("LORAFORGE_SGLANG_ACTIVE_PREFILL", "0")
    if active_prefill not in ("0", "1"):
        raise ValueError("LORAFORGE_SGLANG_ACTIVE_PREFILL must be 0 or 1")
    numerics = os.environ.get("LORAFORGE_SGLANG_NUMERICS", "fp32")
    if numerics not in ("fp32", "reference"):
        raise ValueError("LORAFORGE_SGLANG_NUMERICS must be fp32 or reference")
    data = json.loads(Path(os.environ["LORAFORGE_SGLANG_MANIFEST"]).read_text())
    paths = [a.get("path", a.get("source")) for a in data["adapters"]]
    if any(not p for p in paths):
        raise ValueError("every adapter must declare a local path")
    return create_backend(read_rank_catalog(paths), active_prefill=active_prefill == "1", numerics=numerics)
