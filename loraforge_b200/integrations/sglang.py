"""Opt-in SGLang 0.5.22 LoRA backend on the B200 kernels (drop-in for
``loraforge.integrations.sglang``, src/loraforge/integrations/sglang.py:1-246).

Registration is the reference's: the ``sglang.srt.plugins`` entry point calls
``install()``, which does nothing unless ``LORAFORGE_SGLANG=1``; then
``install_sglang_backend()`` points SGLang's ``csgmv`` backend factory at
``get_backend``, refusing to displace anything but SGLang's own factory.
``LORAFORGE_SGLANG_POLICY`` picks the backend inside each worker:

* ``compatible`` - decode batches through the padded-layout BGMV kernels
  (``lora_shrink`` / ``lora_expand``) on SGLang's own buffers and slot ranks;
* ``rank-aware`` - decode A through the retained-rank row shrink (columns packed at
  s*r of each slot's rank), B through SGLang's chunked SGMV expand;
* ``fleet`` - the retained-rank fleet backend (``_sglang_fleet``): fused
  shrink/expand kernels for QKV and gate/up, row-form kernels for the others.

Prefill and anything the B200 kernels cannot serve stay with SGLang's kernels.
"""

from __future__ import annotations

import os
from functools import lru_cache
from importlib.metadata import version

SGLANG_VERSION = "0.5.22"
POLICIES = ("compatible", "rank-aware", "fleet")


def _check_version():
    if version("sglang") != SGLANG_VERSION:
        raise RuntimeError(f"LoRAForge SGLang integration requires exactly SGLang {SGLANG_VERSION}")


def _decode_policy():
    policy = os.environ.get("LORAFORGE_SGLANG_POLICY", "compatible")
    if policy not in POLICIES:
        raise ValueError("LORAFORGE_SGLANG_POLICY must be compatible, rank-aware, or fleet")
    return policy


@lru_cache(maxsize=1)
def get_backend():
    """The backend class for this worker's policy (resolved once per process)."""
    _check_version()
    policy = _decode_policy()
    if policy == "fleet":
        from ._sglang_fleet import backend_from_environment

        return backend_from_environment()
    from sglang.srt.lora.backend.chunked_backend import ChunkedSgmvLoRABackend

    return decode_backend(ChunkedSgmvLoRABackend, policy)


def decode_backend(base, policy: str):
    """Subclass ``base`` (SGLang's chunked SGMV backend) with B200 decode kernels."""
    import torch

    from loraforge_b200.ops.gemv import lora_expand, lora_shrink
    from loraforge_b200.ops.grouping import segment_routes
    from loraforge_b200.ops.rowexpand import direct_shrink

    def native_expand(z, weights, info, offsets, max_slice, output, offsets_cpu):
        from sglang.kernels.ops.lora.dense.chunked_sgmv_expand import chunked_sgmv_lora_expand_forward

        return chunked_sgmv_lora_expand_forward(
            x=z, weights=weights, batch_info=info, slice_offsets=offsets,
            slice_offsets_cpu=offsets_cpu, max_slice_size=max_slice, base_output=output,
        )

    class LoRAForgeDecodeBackend(base):
        supports_prefill_cuda_graph = False

        def prepare_lora_batch(self, forward_batch, *args, **kwargs):
            super().prepare_lora_batch(forward_batch, *args, **kwargs)
            self._loraforge_decode = forward_batch.forward_mode.is_decode()
            self._loraforge_routes = None

        def _use_decode(self, x, pruned=None):
            info = self.batch_info
            return (
                getattr(self, "_loraforge_decode", False)
                and pruned is None
                and x.shape[0] > 0
                and info is not None
                and info.req_weight_indices is not None
            )

        def _routes(self, tokens):
            # Per-token slots from SGLang's segment table, computed on the device once
            # per batch (and inside the graph when captured).
            if self._loraforge_routes is None or self._loraforge_routes.numel() != tokens:
                info = self.batch_info
                count = getattr(self, "_loraforge_count", None)
                if count is None:
                    count = self._loraforge_count = torch.zeros(1, dtype=torch.int32, device=info.seg_indptr.device)
                segments = info.weight_indices.shape[0] if info.use_cuda_graph else info.num_segments
                count.fill_(segments)
                self._loraforge_routes = segment_routes(
                    info.seg_indptr, info.weight_indices, info.permutation, count, tokens
                )
            return self._loraforge_routes

        def _shrink(self, x, weights, slices=1):
            info = self.batch_info
            if policy == "rank-aware":
                capacity = weights.shape[1] // slices
                if x.dtype == torch.bfloat16 and x.is_contiguous() and capacity <= 64:
                    z = torch.empty((x.shape[0], weights.shape[1]), dtype=x.dtype, device=x.device)
                    return direct_shrink(x, weights, z, self._routes(x.shape[0]), info.lora_ranks, slices,
                                         capacity)
                from sglang.kernels.ops.lora.dense.chunked_sgmv_shrink import chunked_sgmv_lora_shrink_forward

                return chunked_sgmv_lora_shrink_forward(x, weights, info, slices)
            return lora_shrink(x, weights, info.lora_ranks, info.req_weight_indices, slices)

        def _expand(self, z, weights, offsets, max_slice, output, offsets_cpu=None):
            info = self.batch_info
            if policy == "rank-aware" and z.dtype == torch.bfloat16:
                return native_expand(z, weights, info, offsets, max_slice, output, offsets_cpu)
            return lora_expand(z, weights, info.lora_ranks, info.scalings, info.req_weight_indices,
                               offsets, max_slice, output)

        def run_lora_a_sgemm(self, x, weights, pruned_batch_info=None, stack_num=1, *args, **kwargs):
            if self._use_decode(x, pruned_batch_info):
                return self._shrink(x, weights, stack_num)
            return super().run_lora_a_sgemm(x, weights, pruned_batch_info, stack_num, *args, **kwargs)

        def run_lora_b_sgemm(self, x, weights, output_offset, base_output=None, pruned_batch_info=None,
                             *args, **kwargs):
            if self._use_decode(x, pruned_batch_info):
                return self._expand(x, weights, output_offset, weights.shape[-2], base_output,
                                    kwargs.get("output_offset_cpu"))
            return super().run_lora_b_sgemm(x, weights, output_offset, base_output, pruned_batch_info,
                                            *args, **kwargs)

        def run_qkv_lora(self, x, qkv_lora_a, qkv_lora_b, output_offset, max_qkv_out_dim, base_output=None,
                         n_slices=3, *args, **kwargs):
            if self._use_decode(x):
                return self._expand(self._shrink(x, qkv_lora_a, n_slices), qkv_lora_b, output_offset,
                                    max_qkv_out_dim, base_output, kwargs.get("output_offset_cpu"))
            return super().run_qkv_lora(x, qkv_lora_a, qkv_lora_b, output_offset, max_qkv_out_dim,
                                        base_output, n_slices, *args, **kwargs)

        def run_gate_up_lora(self, x, gate_up_lora_a, gate_up_lora_b, output_offset, base_output=None,
                             *args, **kwargs):
            if self._use_decode(x):
                return self._expand(self._shrink(x, gate_up_lora_a, 2), gate_up_lora_b, output_offset,
                                    gate_up_lora_b.shape[-2] // 2, base_output, kwargs.get("output_offset_cpu"))
            return super().run_gate_up_lora(x, gate_up_lora_a, gate_up_lora_b, output_offset, base_output,
                                            *args, **kwargs)

    return LoRAForgeDecodeBackend


def install_sglang_backend():
    """Route SGLang's ``csgmv`` backend to ``get_backend`` in this process (repeatable).

    Refuses to overwrite a factory other than SGLang's own.  SGLang keeps owning its
    fixed-address buffers, routing updates, loader synchronisation and graphs.
    """
    _check_version()
    from sglang.srt.lora.backend.lora_registry import LORA_SUPPORTED_BACKENDS

    current = LORA_SUPPORTED_BACKENDS.get("csgmv")
    if current is get_backend:
        return
    if (
        getattr(current, "__module__", None) != "sglang.srt.lora.backend.lora_registry"
        or getattr(current, "__name__", None) != "create_triton_csgmv_backend"
    ):
        raise RuntimeError("csgmv is already owned by another plugin")
    LORA_SUPPORTED_BACKENDS["csgmv"] = get_backend


def install():
    """``sglang.srt.plugins`` entry point: inert unless ``LORAFORGE_SGLANG=1``."""
    if os.environ.get("LORAFORGE_SGLANG") == "1":
        install_sglang_backend()
