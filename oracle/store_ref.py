"""CPU-tier LRU oracle: restatement of the in-memory adapter LRU of
src/polylora/store.py (CpuAdapterStore) over plain Python state, without the
disk tier: get/touch (store.py:184-199), set_eviction_exclusions
(store.py:201-202), add_adapter (store.py:207-219) and _evict_if_needed
(store.py:425-436).  Test infrastructure only."""

from __future__ import annotations

from collections import OrderedDict


class CpuLru:
    def __init__(self, max_adapters: int | None, base: str = "__base__") -> None:
        if max_adapters is not None and max_adapters < 1:
            raise ValueError("max_adapters must be at least 1")
        self.max_adapters = max_adapters
        self.base = base
        self.adapters: OrderedDict[str, None] = OrderedDict()
        self.exclusions: set[str] = set()

    def get(self, adapter_id: str) -> None:
        if adapter_id == self.base:
            raise KeyError(f"Base adapter {adapter_id!r} has no LoRA weights")
        if adapter_id not in self.adapters:
            raise KeyError(f"Unknown LoRA adapter id: {adapter_id}")
        self.touch(adapter_id)

    def touch(self, adapter_id: str) -> None:
        if adapter_id in self.adapters:
            self.adapters.move_to_end(adapter_id)

    def set_eviction_exclusions(self, adapter_ids: set[str]) -> None:
        self.exclusions = {a for a in adapter_ids if a != self.base}

    def add_adapter(self, adapter_id: str) -> None:
        if adapter_id == self.base:
            raise ValueError(f"{self.base!r} is reserved for base-only rows")
        self.adapters[adapter_id] = None
        self.adapters.move_to_end(adapter_id)
        self._evict_if_needed({adapter_id})

    def _evict_if_needed(self, exclude: set[str]) -> None:
        if self.max_adapters is None:
            return
        exclude = exclude | self.exclusions
        while len(self.adapters) > self.max_adapters:
            for a in list(self.adapters):
                if a in exclude:
                    continue
                self.adapters.pop(a)
                break
            else:
                raise RuntimeError("No evictable CPU LoRA adapter is available")
