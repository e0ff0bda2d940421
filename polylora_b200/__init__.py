"""polylora_b200: batched multi-adapter LoRA inference on B200 (sm_100a).

Drop-in for the reference package's public API (same nine names); the LoRA
math runs in the native library ``libpolylora_b200.so`` (include/polylora_b200.h).
"""

from .cache import GpuAdapterCache
from .config import CustomLoraConfig, PolyLoraConfig
from .context import LoraBatchContext
from .layers import MultiLoraLinear
from .model import CustomPeftModel, PolyLoraModel
from .store import CpuAdapterStore, DiskAdapterCache

__all__ = [
    "CpuAdapterStore",
    "CustomLoraConfig",
    "CustomPeftModel",
    "DiskAdapterCache",
    "GpuAdapterCache",
    "LoraBatchContext",
    "MultiLoraLinear",
    "PolyLoraConfig",
    "PolyLoraModel",
]
