"""vLLM 0.26.0 plugin: dense-linear LoRA decode on the B200 BGMV kernels.

Drop-in for ``loraforge.integrations.vllm`` (src/loraforge/integrations/vllm.py:1-154):
the same entry points (``register`` for ``vllm.general_plugins``, ``install_vllm_backend``)
and the same refusals.  Importing this module loads neither torch nor vLLM.

Design
------
What is taken over.  vLLM's ``PunicaWrapperGPU.add_lora_linear``, one call per LoRA'd
linear layer, when all of these hold: a decode step (``is_prefill`` false), the engine
specialises its graphs on the active-LoRA count (``lora_config.specialize_active_lora``),
the caller passes no ``buffer`` and no keyword other than ``add_inputs``, and the LoRA
rank (A's row count) is 1..256.  Any other call goes to the method that was installed
before, unchanged.

What runs.  One ``torch.library`` custom op (so compiled and captured graphs treat the call
as an opaque mutation of ``y``): ``vllm_gemv.shrink`` writes the FP32 intermediate with the
scale applied, ``vllm_gemv.expand`` adds it into ``y`` with one rounding.  Both sum in a
fixed order, so a decode step gives the same bits every time (the atomics-based split-K of
the stock kernels does not).  The op decides per captured graph from vLLM's host-side
metadata (its no-LoRA flag and active-LoRA count): with no LoRA it does nothing; with more
than ``tokens_per_lora`` tokens per active LoRA it hands the batch to vLLM's own kernels,
whose grouped tiles suit large batches better than a per-token BGMV.

How conflicts are found.  Installation is per worker process and remembered as (the
method installed, its threshold).  Installing again with the same threshold is a no-op;
a different threshold, or finding another method where ours was put, is a conflict; a
method that does not come from vLLM's own module is a foreign backend and is not wrapped.
"""

from __future__ import annotations

import os
from functools import lru_cache
from importlib.metadata import version
from threading import RLock

from loraforge_b200.annotations import ExperimentalAPI

VLLM_VERSION = "0.26.0"
_VLLM_MODULE = "vllm.lora.punica_wrapper.punica_gpu"
_MAX_RANK = 256
_lock = RLock()
_installed = None  # (installed method, tokens_per_lora) once this worker is patched


def _engine_kernels():
    """vLLM's stock shrink / expand (the engine's own path for large batches)."""
    from vllm.lora.ops.triton_ops.lora_expand_op import _lora_expand
    from vllm.lora.ops.triton_ops.lora_shrink_op import _lora_shrink

    return _lora_shrink, _lora_expand


@lru_cache(maxsize=1)
def _operator():
    """Register (once) and return the custom op that performs one layer's LoRA delta."""
    import torch

    from loraforge_b200.ops.vllm_gemv import expand, shrink

    def small_batch(tokens, active_loras, threshold):
        return tokens <= threshold * max(1, active_loras)

    @torch.library.custom_op("loraforge_b200::vllm_linear", mutates_args=("y",))
    def vllm_linear(
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
        # `no_lora` and `active` live on the host; a captured graph fixes the branch taken.
        if no_lora.item():
            return
        rank = b[0].shape[-1]
        with torch.cuda.device(x.device):
            intermediate = torch.empty((len(a), x.shape[0], rank), dtype=torch.float32, device=x.device)
            if small_batch(x.shape[0], int(active.item()), threshold):
                shrink(x, a, intermediate, routes, scale=scale)
                expand(intermediate, b, y, routes, add=add)
                return
            stock_shrink, stock_expand = _engine_kernels()
            metadata = (routes, sorted_tokens, counts, starts, ids, no_lora, active)
            stock_shrink(x, a, intermediate, *metadata, scale)
            stock_expand(intermediate, b, y, *metadata, offset_start=0, add_inputs=add)

    @vllm_linear.register_fake
    def _vllm_linear_shape(*args, **kwargs):  # mutates y in place, returns nothing
        return None

    return vllm_linear


def _takes_over(wrapper, lora_a_stacked, buffer, kwargs) -> bool:
    """Whether a call of add_lora_linear is one this plugin runs (see the module notes)."""
    return (
        not wrapper.is_prefill
        and bool(wrapper.lora_config.specialize_active_lora)
        and buffer is None
        and not (set(kwargs) - {"add_inputs"})
        and bool(lora_a_stacked)
        and 1 <= lora_a_stacked[0].shape[-2] <= _MAX_RANK
    )


def _patched_method(previous, op, tokens_per_lora):
    def add_lora_linear(self, y, x, lora_a_stacked, lora_b_stacked, scale, output_slices, *, buffer=None,
                        **kwargs):
        if not _takes_over(self, lora_a_stacked, buffer, kwargs):
            return previous(self, y, x, lora_a_stacked, lora_b_stacked, scale, output_slices,
                            buffer=buffer, **kwargs)
        if len({len(lora_a_stacked), len(lora_b_stacked), len(output_slices)}) != 1:
            raise ValueError("slice counts must match")
        if tuple(output_slices) != tuple(b.shape[-2] for b in lora_b_stacked):
            raise ValueError("output slice widths must match B")
        flat_x = x.view(-1, x.shape[-1])
        flat_y = y.view(-1, y.shape[-1])
        op(flat_y, flat_x, list(lora_a_stacked), list(lora_b_stacked), float(scale),
           *self.token_mapping_meta.meta_args(flat_x.shape[0], True), kwargs.get("add_inputs", True),
           tokens_per_lora)

    return add_lora_linear


@ExperimentalAPI(
    reason="Opt-in vLLM 0.26.0 specialized linear decode on sm_100a kernels; synthetic validation only.",
    warn=True,
)
def install_vllm_backend(*, tokens_per_lora: int = 4) -> None:
    """Patch vLLM's ``add_lora_linear`` in this worker; call before the model is built.

    Installing twice with the same ``tokens_per_lora`` does nothing; a different value or a
    method replaced by someone else since raises, and so does a foreign method.
    """
    global _installed
    if type(tokens_per_lora) is not int or tokens_per_lora < 1:
        raise ValueError("tokens_per_lora must be a positive integer")
    if version("vllm") != VLLM_VERSION:
        raise RuntimeError(f"LoRAForge requires exactly vLLM {VLLM_VERSION}")
    from vllm.lora.punica_wrapper.punica_gpu import PunicaWrapperGPU

    with _lock:
        present = PunicaWrapperGPU.add_lora_linear
        if _installed is not None:
            ours, threshold = _installed
            if present is ours and tokens_per_lora == threshold:
                return
            raise RuntimeError("vLLM registration conflicts with existing backend")
        if present.__module__ != _VLLM_MODULE:
            raise RuntimeError("refusing to replace a foreign vLLM backend")
        method = _patched_method(present, _operator(), tokens_per_lora)
        PunicaWrapperGPU.add_lora_linear = method
        _installed = method, tokens_per_lora


@ExperimentalAPI(reason="Environment-gated vLLM 0.26.0 plugin entry point; explicit per-worker activation.")
def register() -> None:
    """``vllm.general_plugins`` entry point; does nothing unless ``LORAFORGE_VLLM=1``."""
    if os.environ.get("LORAFORGE_VLLM") == "1":
        install_vllm_backend()
