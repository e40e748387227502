"""Fixed-address kernel operands of one projection, filled from resident adapters.

The fused operators read, per projection of a layer, a packed A slab
[slots, slices*capacity, width] (slot g's slice s at rows s*k .. s*k+k-1 for the
slot's rank k), a flat compact B store (slot g's [N, bucket_g] block at
b_offsets[g]) and per-slot rank, bucket and scale vectors.  ``ProjectionSlab``
owns all of them at fixed device addresses for its lifetime, so graphs captured
over them stay valid while adapters come and go.  Each slot's B block is reserved
at the capacity's bucket, so any rank up to the capacity fits without moving
another slot; the kernels read only N*bucket_g elements of it, so the HBM traffic
of a call stays compact.  This is the standalone counterpart of ``RetainedLayout``
(which packs inside a serving framework's own padded buffers); it follows the same
packing rules (src/loraforge/runtime/retained.py:146-205).

``load`` takes the slices' ``AdapterModule``s (from ``GPUAdapterSlots.borrow`` or
CPU tensors), casts to BF16 and scatters them on the current stream; a slot whose
slices have different scalings gets one slot scale (the first slice's) with the
other slices' B columns multiplied by their scaling ratio before rounding.
"""

from __future__ import annotations

import re

from .retained import MAX_KERNEL_RANK, bucket_of


def select_modules(modules, layer: int, names) -> list:
    """The module of each name in ``names`` (or None) for ``layer``, matched on the
    PEFT module path ``...layers.<layer>.<...>.<name>``."""
    found = []
    for name in names:
        pattern = re.compile(rf"(?:^|\.)layers\.{layer}\.(?:.*\.)?{re.escape(name)}$")
        hits = [m for m in modules if pattern.search(m.name)]
        if len(hits) > 1:
            raise ValueError(f"several modules match layer {layer} {name}")
        found.append(hits[0] if hits else None)
    return found


class ProjectionSlab:
    """Packed A slab, compact B store and slot metadata for one LoRA projection."""

    def __init__(self, slots: int, width: int, slice_widths, capacity: int, *, device):
        import torch

        slice_widths = tuple(int(w) for w in slice_widths)
        if type(slots) is not int or slots < 1:
            raise ValueError("slots must be a positive integer")
        if not 1 <= len(slice_widths) <= 4 or min(slice_widths) < 1:
            raise ValueError("one to four positive slice widths are required")
        if type(capacity) is not int or not 1 <= capacity <= MAX_KERNEL_RANK:
            raise ValueError(f"capacity must be in 1..{MAX_KERNEL_RANK}")
        if type(width) is not int or width < 8 or width % 8:
            raise ValueError("width must be a positive multiple of 8")
        self.device = torch.device(device)
        self.width, self.slice_widths, self.capacity = width, slice_widths, capacity
        self.num_slices, self.out_width = len(slice_widths), sum(slice_widths)
        self.region = -(-self.out_width * bucket_of(capacity) // 8) * 8  # 8-element aligned blocks
        bf16, dev = torch.bfloat16, self.device
        self.a = torch.zeros(slots, self.num_slices * capacity, width, dtype=bf16, device=dev)
        self.b = torch.zeros(slots * self.region, dtype=bf16, device=dev)
        self.b_offsets = torch.arange(slots, dtype=torch.int64, device=dev) * self.region
        self.b_strides = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.ranks = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.scales = torch.zeros(slots, dtype=torch.float32, device=dev)
        bounds = [0]
        for w in slice_widths:
            bounds.append(bounds[-1] + w)
        self.slice_offsets = torch.tensor(bounds, dtype=torch.int32, device=dev)
        self.loaded: dict[int, dict] = {}

    def _slot(self, slot) -> None:
        if type(slot) is not int or not 0 <= slot < self.a.shape[0]:
            raise ValueError("slot outside slab capacity")

    def load(self, slot: int, modules) -> None:
        """Pack one adapter's slices (a sequence of ``AdapterModule`` or None) into ``slot``."""
        import torch

        self._slot(slot)
        modules = list(modules)
        if len(modules) != self.num_slices:
            raise ValueError("one module (or None) per slice is required")
        live = [m for m in modules if m is not None]
        if not live:
            self.clear(slot)
            return
        for s, m in enumerate(modules):
            if m is None:
                continue
            if m.a.shape[1] != self.width or m.b.shape[0] != self.slice_widths[s] or m.b.shape[1] != m.rank:
                raise ValueError(f"slice {s} factors do not match the projection's shape")
        k = max(m.rank for m in live)
        if k > self.capacity:
            raise ValueError("adapter rank exceeds slab capacity")
        bucket, scale = bucket_of(k), live[0].scaling
        a = torch.zeros(self.num_slices * k, self.width, dtype=torch.bfloat16, device=self.device)
        b = torch.zeros(self.out_width, bucket, dtype=torch.bfloat16, device=self.device)
        row0 = 0
        for s, m in enumerate(modules):
            if m is not None:
                a[s * k : s * k + m.rank] = m.a.to(self.device, torch.bfloat16)
                factor = m.b.to(self.device, torch.float32)
                if m.scaling != scale:
                    factor = factor * (m.scaling / scale)
                b[row0 : row0 + self.slice_widths[s], : m.rank] = factor.to(torch.bfloat16)
            row0 += self.slice_widths[s]
        self.a[slot].zero_()
        self.a[slot, : self.num_slices * k] = a
        start = slot * self.region
        self.b[start : start + self.out_width * bucket] = b.reshape(-1)
        self.ranks[slot] = k
        self.b_strides[slot] = bucket
        self.scales[slot] = scale
        self.loaded[slot] = dict(rank=k, bucket=bucket, scale=scale, modules=[m and m.name for m in modules])

    def clear(self, slot: int) -> None:
        """Make ``slot`` inert: its segments are skipped by the kernels."""
        self._slot(slot)
        self.ranks[slot] = 0
        self.b_strides[slot] = 0
        self.scales[slot] = 0.0
        self.loaded.pop(slot, None)

    def operands(self) -> dict:
        """A and the metadata keywords of ``lora_shrink_expand`` (routing not included)."""
        return dict(
            a=self.a, b=self.b, b_offsets=self.b_offsets, b_strides=self.b_strides, ranks=self.ranks,
            scales=self.scales, slice_offsets=self.slice_offsets, num_slices=self.num_slices,
        )
