"""Compact B store and per-slot rank metadata for one fused projection of a layer.

Drop-in for ``loraforge.runtime.retained`` (src/loraforge/runtime/retained.py:17-205):
``read_rank_catalog``, ``effective_rank`` and ``RetainedLayout`` with the same region
arithmetic, per-slot fields and error messages, so the reference's known-answer
sequence (tests/test_retained_layout.py:24-61) reproduces bit for bit.

The layout sits beside a serving framework's padded per-slot buffers
(A [slots, slices*capacity, width], B [slots, width_out, capacity]).  At
construction every checkpoint of a frozen catalog gets a fixed region of the
compact store: its effective rank k (the largest retained rank of the
projection's modules in that layer), bucket = next power of two >= k, start
rounded up to 8 elements, width_out*bucket elements when 1 <= k <= 64.  Loading a
checkpoint into a slot after the framework's own load

* repacks the slot's A rows in place from stride ``checkpoint_rank`` to stride k
  (slice s moves to rows s*k .. s*k+k-1), which is the A layout the shrink
  kernels read;
* copies the slot's first k B columns into the checkpoint's region (zero padding
  up to the bucket), the compact B the expand kernels read;
* writes the slot's rank classes: ``rank``, ``supported`` (k <= 64), ``unsupported``
  (k > 64), ``low`` (k <= 16), ``high`` (k > 16), ``bucket``, ``boff``.

Every tensor keeps its address for the layout's lifetime, so graphs captured over
it stay valid across loads.  Loads are outside graph capture and must not race
consumers; the caller orders them.
"""

from __future__ import annotations

import json
import re
from pathlib import Path

# SGLang's fused projections and the checkpoint modules each one stacks.
FUSED_TARGETS = {
    "qkv_proj": ("qkv_proj", "q_proj", "k_proj", "v_proj"),
    "gate_up_proj": ("gate_up_proj", "gate_proj", "up_proj"),
    "in_proj_qkvz": ("in_proj_qkvz", "in_proj_qkv", "in_proj_q", "in_proj_k", "in_proj_v", "in_proj_z"),
    "in_proj_ba": ("in_proj_ba", "in_proj_b", "in_proj_a"),
}
MAX_KERNEL_RANK = 64
LOW_RANK = 16
_FIELDS = ("rank", "supported", "unsupported", "low", "high", "bucket")


def _header(path: Path) -> dict:
    with path.open("rb") as handle:
        length = int.from_bytes(handle.read(8), "little")
        if not 2 <= length <= 64 * 1024 * 1024:
            raise ValueError("invalid safetensors header length")
        return json.loads(handle.read(length))


def read_rank_catalog(paths) -> dict[str, dict[str, int]]:
    """{resolved checkpoint path: {A tensor key: retained rank}} for padded PEFT exports.

    Every checkpoint must use one global rank (no per-module rank/alpha patterns,
    no rsLoRA) with every A/B pair at that rank.  An optional ``compression.json``
    (``{"module_ranks": {A key: k}}``) lowers per-module ranks; it must name exactly
    the A tensors, and the factor columns beyond k must be zero.
    """
    catalog = {}
    for raw in paths:
        path = Path(raw).resolve()
        config = json.loads((path / "adapter_config.json").read_text())
        rank = config["r"]
        if type(rank) is not int or rank < 1:
            raise ValueError("invalid checkpoint rank")
        if config.get("rank_pattern") or config.get("alpha_pattern") or config.get("use_rslora"):
            raise ValueError("convert per-module rank/scaling to SGLang padding first")
        header = _header(path / "adapter_model.safetensors")
        ranks = {}
        for key, info in header.items():
            if not key.endswith(".lora_A.weight"):
                continue
            partner = header.get(key[: -len(".lora_A.weight")] + ".lora_B.weight")
            if len(info["shape"]) != 2 or info["shape"][0] != rank or partner is None or partner["shape"][-1] != rank:
                raise ValueError("native SGLang requires padded global-rank tensors")
            ranks[key] = rank
        if not ranks:
            raise ValueError("no linear LoRA A/B pairs found")
        metadata = path / "compression.json"
        if metadata.exists():
            declared = json.loads(metadata.read_text())["module_ranks"]
            if declared.keys() != ranks.keys():
                raise ValueError("retained rank metadata must cover exactly the A tensors")
            for key, k in declared.items():
                if type(k) is not int or not 0 < k <= rank:
                    raise ValueError("retained rank exceeds checkpoint rank")
            _check_zero_tails(path, {key: k for key, k in declared.items() if k < rank})
            ranks.update(declared)
        catalog[str(path)] = ranks
    if not catalog:
        raise ValueError("a nonempty frozen adapter catalog is required")
    return catalog


def _check_zero_tails(path: Path, lowered: dict[str, int]) -> None:
    # A declared rank below the padded one is only valid if it drops zeros.
    if not lowered:
        return
    from safetensors import safe_open

    with safe_open(str(path / "adapter_model.safetensors"), framework="pt", device="cpu") as weights:
        for key, k in lowered.items():
            a = weights.get_tensor(key)
            b = weights.get_tensor(key.replace(".lora_A.weight", ".lora_B.weight"))
            if a[k:].count_nonzero().item() or b[:, k:].count_nonzero().item():
                raise ValueError("retained-rank metadata truncates nonzero padded factors")


def effective_rank(ranks: dict[str, int], name: str, layer: int) -> int:
    """Largest retained rank among the modules fused into projection ``name`` of ``layer``."""
    targets = set(FUSED_TARGETS.get(name, (name,)))
    layer_tag = re.compile(rf"\.layers\.{layer}\.")
    return max(
        (r for key, r in ranks.items() if layer_tag.search(key) and key.split(".")[-3] in targets),
        default=0,
    )


def bucket_of(k: int) -> int:
    """Smallest power of two >= max(k, 1)."""
    return 1 << (max(1, k) - 1).bit_length()


class RetainedLayout:
    """Fixed compact B regions and per-slot rank metadata for one fused projection."""

    def __init__(self, a, b, name: str, layer: int, catalog: dict[str, dict[str, int]]):
        import torch

        if a.ndim != 3 or b.ndim != 3 or a.dtype != torch.bfloat16 or b.dtype != a.dtype or a.device != b.device:
            raise ValueError("retained layout requires matching BF16 3D buffers")
        slots, width_out, capacity = b.shape
        if a.shape[0] != slots or capacity < 1 or a.shape[1] % capacity or not 1 <= a.shape[1] // capacity <= 4:
            raise ValueError("invalid fused A/B capacity")
        if not (a.is_contiguous() and b.is_contiguous()):
            raise ValueError("native buffers must be contiguous")
        self.a, self.b, self.name, self.layer = a, b, name, layer
        self.capacity, self.slices = capacity, a.shape[1] // capacity
        self.regions: dict[str, tuple[int, int, int]] = {}
        end = 0
        for path, ranks in catalog.items():
            k = effective_rank(ranks, name, layer)
            if k > capacity:
                raise ValueError("effective rank exceeds native capacity")
            end = -(-end // 8) * 8
            self.regions[path] = (end, bucket_of(k), k)
            if 0 < k <= MAX_KERNEL_RANK:
                end += width_out * bucket_of(k)
        device = b.device
        self.store = torch.zeros(max(1, end), dtype=b.dtype, device=device)
        for field in _FIELDS:
            setattr(self, field, torch.zeros(slots, dtype=torch.int32, device=device))
        self.boff = torch.zeros(slots, dtype=torch.int64, device=device)
        ks = [k for _, _, k in self.regions.values()]
        self.has_high = any(k > LOW_RANK for k in ks)
        self.has_unsupported = any(k > MAX_KERNEL_RANK for k in ks)
        self.max_rank = max([1] + [min(MAX_KERNEL_RANK, bucket) for _, bucket, _ in self.regions.values()])
        self.loaded: dict[int, dict] = {}

    def validate_load(self, path, checkpoint_rank: int) -> None:
        """Refuse, before any buffer changes, a checkpoint this layout cannot hold."""
        if path is None:
            return
        if path not in self.regions:
            raise ValueError("checkpoint is absent from frozen rank catalog")
        if not self.regions[path][2] <= checkpoint_rank <= self.capacity:
            raise ValueError("checkpoint rank does not fit retained layout")

    def load(self, path, slot: int, checkpoint_rank: int = 0) -> None:
        """Repack the slot's A, fill its B region and metadata (``path`` None clears the slot)."""
        import torch

        self.validate_load(path, checkpoint_rank)
        if not 0 <= slot < self.b.shape[0]:
            raise ValueError("slot out of range")
        offset, bucket, k = (0, 0, 0) if path is None else self.regions[path]
        if k and k != checkpoint_rank:
            rows = torch.tensor(
                [s * checkpoint_rank + j for s in range(self.slices) for j in range(k)], device=self.a.device
            )
            self.a[slot, : self.slices * k] = self.a[slot].index_select(0, rows)
        if 0 < k <= MAX_KERNEL_RANK:
            region = self.store[offset : offset + self.b.shape[1] * bucket].view(self.b.shape[1], bucket)
            region.zero_()
            region[:, :k] = self.b[slot, :, :k]
        values = dict(
            rank=k,
            supported=k if k <= MAX_KERNEL_RANK else 0,
            unsupported=k if k > MAX_KERNEL_RANK else 0,
            low=k if k <= LOW_RANK else 0,
            high=k if k > LOW_RANK else 0,
            bucket=bucket,
            boff=offset,
        )
        for field, value in values.items():
            getattr(self, field)[slot] = value
        self.loaded[slot] = dict(path=path, rank=k, checkpoint_rank=checkpoint_rank)

    def kernel_operands(self, *, rank_class: str = "supported") -> dict:
        """B store and per-slot metadata as keyword arguments of the fused operators.

        ``rank_class`` ``"supported"`` serves every slot of rank 1..64 (all the B200
        kernels take); ``"low"`` only ranks 1..16.  Pass ``self.a`` as A; segments of
        slots outside the class are skipped.  The tensors are the layout's own, so a
        graph captured over them sees every later load.
        """
        if rank_class not in ("supported", "low"):
            raise ValueError("rank_class must be supported or low")
        return dict(b=self.store, b_offsets=self.boff, b_strides=self.bucket, ranks=getattr(self, rank_class))
