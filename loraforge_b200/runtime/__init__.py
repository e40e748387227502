"""Adapter residency (drop-in for ``loraforge.runtime``): CPU and GPU slot pools,
generation-checked handles, and the compact retained-rank layout."""

from .gpu import GPUAdapterSlots
from .slots import AdapterSlots, SlotHandle

__all__ = ["GPUAdapterSlots", "AdapterSlots", "SlotHandle"]
