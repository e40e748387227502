"""PEFT linear-LoRA checkpoints (drop-in for ``loraforge.adapters``' loader)."""

from .peft import AdapterModule, PeftAdapter, load_peft_adapter, write_manifest

__all__ = ["AdapterModule", "PeftAdapter", "load_peft_adapter", "write_manifest"]
