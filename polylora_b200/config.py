"""Configuration of the multi-adapter wrapper.

Same fields, defaults and validation messages as the reference's
``PolyLoraConfig`` (src/polylora/config.py:5-32) so configs port unchanged.
``use_triton_kernels`` is kept for compatibility: here it selects the native
sm_100a kernels, and turning it off is rejected at forward time because this
package has no non-CUDA compute path.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path


@dataclass(frozen=True)
class PolyLoraConfig:
    max_gpu_adapters: int
    max_rank: int
    target_modules: list[str] | None = None
    max_cpu_adapters: int | None = None
    disk_cache_dir: str | Path | None = None
    max_disk_adapters: int | None = None
    base_adapter_id: str = "__base__"
    enforce_right_padding: bool = True
    use_triton_kernels: bool = True
    # threads of the CPU tier's disk prefetch (PolyLoraModel.prefetch); None: 1.
    # No counterpart in the reference.
    prefetch_workers: int | None = None
    # where enforce_right_padding checks the mask: "host" compares it at once
    # (the reference's check, which waits for the device), "device" enqueues a
    # library kernel that records a violation in the device status word, read
    # by PolyLoraModel.raise_for_device_status().  No counterpart in the reference.
    right_padding_check: str = "host"

    def __post_init__(self) -> None:
        checks = (
            (self.max_gpu_adapters < 1, "max_gpu_adapters must be at least 1"),
            (
                self.max_cpu_adapters is not None and self.max_cpu_adapters < self.max_gpu_adapters,
                "max_cpu_adapters must be at least max_gpu_adapters",
            ),
            (
                self.max_disk_adapters is not None and self.max_disk_adapters < 1,
                "max_disk_adapters must be at least 1",
            ),
            (
                self.max_disk_adapters is not None and self.disk_cache_dir is None,
                "disk_cache_dir must be set when max_disk_adapters is set",
            ),
            (self.max_rank < 1, "max_rank must be at least 1"),
            (
                self.target_modules is not None and not self.target_modules,
                "target_modules must not be empty when provided",
            ),
            (self.right_padding_check not in ("host", "device"), 'right_padding_check must be "host" or "device"'),
        )
        for failed, message in checks:
            if failed:
                raise ValueError(message)

    @property
    def use_native_kernels(self) -> bool:
        return self.use_triton_kernels


CustomLoraConfig = PolyLoraConfig
