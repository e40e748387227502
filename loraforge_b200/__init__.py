"""B200-native (sm_100a) multi-LoRA shrink/expand path with LoRAForge's operator API.

Importing the package loads neither torch nor the CUDA library; both are loaded
on the first operator call.
"""

__version__ = "0.1.0"
