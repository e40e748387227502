"""GPU tensor operators (drop-in for ``loraforge.ops``), loaded without touching a device."""

from .gemv import lora_expand, lora_shrink
from .lora_rows import row_expand, row_shrink

__all__ = ["lora_shrink", "lora_expand", "row_shrink", "row_expand"]
