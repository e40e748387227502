"""Opt-in vLLM 0.26.0 linear-LoRA decode on the B200 kernels (drop-in for
``loraforge.integrations.vllm``, src/loraforge/integrations/vllm.py:1-154).

``register`` is the ``vllm.general_plugins`` entry point and does nothing unless
``LORAFORGE_VLLM=1``.  ``install_vllm_backend`` wraps
``PunicaWrapperGPU.add_lora_linear`` in each worker: specialised dense-linear decode
batches whose LoRA rank is 1..256 go through one ``torch.library`` custom op that
runs the padded-slot BGMV kernels (``vllm_gemv.shrink`` with the scale applied in
FP32, then ``vllm_gemv.expand`` with one rounding); everything else (prefill,
unspecialised execution, extra keyword contracts, larger batches per active LoRA
than ``tokens_per_lora``) stays with vLLM's own kernels.  Unlike the atomics-based
split-K the reference pairs with, the B200 shrink sums K in a fixed order, so a
decode step is bitwise repeatable.  Importing this module loads neither torch nor
vLLM.
"""

from __future__ import annotations

import os
from functools import lru_cache
from importlib.metadata import version
from threading import RLock

from loraforge_b200.annotations import ExperimentalAPI

VLLM_VERSION = "0.26.0"
_lock = RLock()
_installed = None


@lru_cache(maxsize=1)
def _operator():
    import torch

    from loraforge_b200.ops.vllm_gemv import expand, shrink

    @torch.library.custom_op("loraforge_b200::vllm_linear", mutates_args=("y",))
    def linear(
        y: torch.Tensor,
        x: torch.Tensor,
        a: list[torch.Tensor],
        b: list[torch.Tensor],
        scale: float,
        routes: torch.Tensor,
        sorted_tokens: torch.Tensor,
        counts: torch.Tensor,
        starts: torch.Tensor,
        ids: torch.Tensor,
        no_lora: torch.Tensor,
        active: torch.Tensor,
        add: bool,
        threshold: int,
    ) -> None:
        # no_lora / active are vLLM's CPU metadata; each captured graph specialises on
        # them, while the routing itself stays on the device.
        if no_lora.item():
            return
        with torch.cuda.device(x.device):
            z = torch.empty((len(a), x.shape[0], b[0].shape[-1]), device=x.device, dtype=torch.float32)
            if x.shape[0] <= threshold * max(1, int(active.item())):
                shrink(x, a, z, routes, scale=scale)
                expand(z, b, y, routes, add=add)
            else:
                from vllm.lora.ops.triton_ops.lora_expand_op import _lora_expand
                from vllm.lora.ops.triton_ops.lora_shrink_op import _lora_shrink

                meta = (routes, sorted_tokens, counts, starts, ids, no_lora, active)
                _lora_shrink(x, a, z, *meta, scale)
                _lora_expand(z, b, y, *meta, offset_start=0, add_inputs=add)

    @linear.register_fake
    def _(*args, **kwargs):
        return None

    return linear


@ExperimentalAPI(
    reason="Opt-in vLLM 0.26.0 specialized linear decode on sm_100a kernels; synthetic validation only.",
    warn=True,
)
def install_vllm_backend(*, tokens_per_lora: int = 4) -> None:
    """Wrap vLLM's ``add_lora_linear`` in this worker (before model construction).

    Repeatable with the same threshold; refuses to replace a foreign backend or to
    change an installed one.
    """
    global _installed
    if type(tokens_per_lora) is not int or tokens_per_lora < 1:
        raise ValueError("tokens_per_lora must be a positive integer")
    if version("vllm") != VLLM_VERSION:
        raise RuntimeError(f"LoRAForge requires exactly vLLM {VLLM_VERSION}")
    from vllm.lora.punica_wrapper.punica_gpu import PunicaWrapperGPU

    with _lock:
        current = PunicaWrapperGPU.add_lora_linear
        if _installed is not None:
            patched, threshold = _installed
            if current is not patched or tokens_per_lora != threshold:
                raise RuntimeError("vLLM registration conflicts with existing backend")
            return
        if current.__module__ != "vllm.lora.punica_wrapper.punica_gpu":
            raise RuntimeError("refusing to replace a foreign vLLM backend")
        op = _operator()

        def add_lora_linear(self, y, x, lora_a_stacked, lora_b_stacked, scale, output_slices, *, buffer=None,
                            **kwargs):
            if (
                self.is_prefill
                or not self.lora_config.specialize_active_lora
                or buffer is not None
                or set(kwargs) - {"add_inputs"}
                or not lora_a_stacked
                or not 1 <= lora_a_stacked[0].shape[-2] <= 256
            ):
                return current(self, y, x, lora_a_stacked, lora_b_stacked, scale, output_slices,
                               buffer=buffer, **kwargs)
            if not len(lora_a_stacked) == len(lora_b_stacked) == len(output_slices):
                raise ValueError("slice counts must match")
            if tuple(b.shape[-2] for b in lora_b_stacked) != tuple(output_slices):
                raise ValueError("output slice widths must match B")
            x2, y2 = x.view(-1, x.shape[-1]), y.view(-1, y.shape[-1])
            op(y2, x2, list(lora_a_stacked), list(lora_b_stacked), float(scale),
               *self.token_mapping_meta.meta_args(x2.shape[0], True), kwargs.get("add_inputs", True),
               tokens_per_lora)

        PunicaWrapperGPU.add_lora_linear = add_lora_linear
        _installed = add_lora_linear, tokens_per_lora


@ExperimentalAPI(reason="Environment-gated vLLM 0.26.0 plugin entry point; explicit per-worker activation.")
def register() -> None:
    """``vllm.general_plugins`` entry point: inert unless ``LORAFORGE_VLLM=1``."""
    if os.environ.get("LORAFORGE_VLLM") == "1":
        install_vllm_backend()
